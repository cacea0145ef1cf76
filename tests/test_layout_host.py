"""Host-side planning code of the library (``ae_b200/csrc/layout.h``), compiled with g++ on
the CPU: the split-K choice of the unit-queue simulation for the benchmark shapes, the
workspace size behind the no-allocation entry point's documented limit, and the exchange
arena layout.  No GPU needed."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include "layout.h"
#include <cstdio>
int main() {
  const int sms = 148;
  struct C { const char* n; int E, H, I, Tk; } cs[] = {
    {"c2_t256", 8, 4096, 14336, 512}, {"c5_t512", 8, 6144, 16384, 1024},
    {"c2_t16", 8, 4096, 14336, 32}, {"c3", 60, 2048, 1408, 512}};
  for (auto& c : cs) std::printf("split %s %d\n", c.n, smb::choose_splits(c.E, c.H, c.I, c.Tk, sms));
  // gate/up K slices: one Mixtral expert on each of 8 ranks (512 exchange rows), two on
  // each of 4, and the single-GPU verify batch
  std::printf("slices ep8 %d\n", smb::choose_plan(1, 4096, 14336, 512, sms).ks1);
  std::printf("slices ep4 %d\n", smb::choose_plan(2, 4096, 14336, 512, sms).ks1);
  std::printf("slices c2_t256 %d\n", smb::choose_plan(8, 4096, 14336, 512, sms).ks1);
  const smb::WsLayout ep8 = smb::make_ws_layout(512, 1, 1, 4096, 14336, 2, smb::choose_plan(1, 4096, 14336, 512, sms));
  std::printf("ep8_gu_bytes %zu\n", ep8.total - ep8.gu);
  std::printf("ep8_ndone %d\n", ep8.ndone);
  const smb::WsLayout pf = smb::make_ws_layout(2048, 8, 2, 4096, 14336, 2, smb::choose_plan(8, 4096, 14336, 4096, sms));
  std::printf("prefill_ntc %d\n", pf.ntc);
  int first_over = -1;
  for (int T = 1; T <= 1024 && first_over < 0; ++T) {
    const smb::FfnPlan p = smb::choose_plan(8, 4096, 14336, 2 * T, sms);
    if (smb::make_ws_layout(T, 8, 2, 4096, 14336, 2, p).total > (64u << 20)) first_over = T;
  }
  std::printf("noalloc_first_over %d\n", first_over);
  const smb::EpArena a = smb::make_ep_arena(8, 64, 4096, 2);
  std::printf("arena %zu %zu %zu %zu\n", a.flags, a.recv, a.back, a.total);
  return 0;
}
"""


@pytest.fixture(scope="module")
def planning():
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "plan.cpp")
        exe = os.path.join(d, "plan")
        with open(src, "w") as f:
            f.write(PROGRAM)
        subprocess.run([gxx, "-O2", "-std=c++17", "-I", os.path.join(ROOT, "ae_b200", "csrc"), src, "-o", exe],
                       check=True, capture_output=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    res = {}
    for line in out.splitlines():
        parts = line.split()
        res[" ".join(parts[:-1]) if parts[0] in ("split", "slices") else parts[0]] = \
            parts[1:] if parts[0] == "arena" else int(parts[-1])
    return res


def test_split_k_choices_match_measured_optima(planning):
    # graph-replay sweeps on B200: Mixtral-8x7B T=256 best at S=2, Mixtral-8x22B T=512 at S=3
    assert planning["split c2_t256"] == 2
    assert planning["split c5_t512"] == 3
    assert 1 <= planning["split c3"] <= 2
    assert planning["split c2_t16"] >= 8


def test_gate_up_slices_only_when_units_underfill_the_gpu(planning):
    # one Mixtral-8x7B expert gives 112 gate/up units for 148 SMs: two K slices (224 units)
    assert planning["slices ep8"] == 2
    assert planning["slices ep4"] == 1
    assert planning["slices c2_t256"] == 1
    # the first slice's fp32 gate/up partials: [rows = 512 + 64, 2 * 14336] floats
    assert planning["ep8_gu_bytes"] == 576 * 2 * 14336 * 4
    # counters: 2 + E*S*ntc + E*m1*ntc with ntc = 2 token tiles of 256 rows bound
    assert planning["ep8_ndone"] >= 2 + 112 * 2
    assert planning["prefill_ntc"] == 16


def test_noalloc_limit_statement(planning):
    # include/ae_b200.h: Mixtral-8x7B shapes fit the 64 MiB scratch for every T <= 448
    assert planning["noalloc_first_over"] == 449


def test_exchange_arena_offsets(planning):
    flags, recv, back, total = (int(v) for v in planning["arena"])
    assert (flags, recv) == (256, 1024)
    assert back == 1024 + 8 * 65 * 4096 * 2
    assert total == back + 8 * 64 * 4096 * 2
