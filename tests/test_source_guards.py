"""Source guards (CPU): the repository's code must not name the cluster-wide TMA or bulk
load variants, nor the batched host-device copy calls, anywhere (comments included); runs
on several GPUs are refused while a travelling source file does.  The patterns are built
from pieces so that this file does not name them either."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CODE_EXT = (".py", ".cu", ".cuh", ".h", ".hpp", ".cpp", ".c", ".sh")
SKIP_DIRS = {".git", "_work", "gpurun_out", "__pycache__", ".pytest_cache", ".hypothesis", "baseline"}

PATTERNS = [
    re.compile("multi" + "cast"),
    re.compile("cuda" + "Memcpy" + "Batch" + "Async"),
    re.compile("cuda" + "Memcpy3D" + "Batch" + "Async"),
    re.compile("cu" + "Memcpy" + "Batch" + "Async"),
    re.compile("cu" + "Memcpy3D" + "Batch" + "Async"),
]


def _code_files():
    for dirpath, dirnames, files in os.walk(ROOT):
        dirnames[:] = [d for d in dirnames if d not in SKIP_DIRS]
        for f in files:
            if f.endswith(CODE_EXT):
                yield os.path.join(dirpath, f)


def test_no_forbidden_names_in_code():
    hits = []
    for path in _code_files():
        with open(path, errors="replace") as fh:
            for n, line in enumerate(fh, 1):
                for p in PATTERNS:
                    if p.search(line):
                        hits.append(f"{os.path.relpath(path, ROOT)}:{n}")
    assert not hits, hits
