"""Expert pages streamed from page-locked host memory while the layer runs
(``ae_b200.streaming.ExpertPageStreamer``: per-page copies + ready flags, the FFN kernel
waits per unit for its page).  Against the fp32 oracle; a second round of copies with new
weights; and a page whose flag nothing raises: the kernel's bounded wait runs out, the
call reports SMB_ERR_DEVICE_TIMEOUT and the context stays usable.
Bars: hidden states max-abs <= 2e-2 and relative-L2 <= 1e-2 against the fp32 oracle."""
import pytest
import torch

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def _host_pages(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(E, 3 * I * H, generator=g) * 0.02).to(torch.bfloat16).pin_memory()


def _inputs(T, E, H, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g).to(torch.bfloat16)
    return x, logits


def _check(out, x, logits, host, pages_of_expert, k):
    w, ids = mo.select_experts(logits, k, True)
    pool = host[torch.as_tensor(pages_of_expert)]  # expert e's weights
    ref = mo.stack_fused_moe(x, pool, torch.arange(len(pages_of_expert)), w, ids, rounding="fp32")
    max_abs, rel = mo.error_metrics(out.float().cpu(), ref)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)


def test_streamed_layer_two_rounds():
    from ae_b200.streaming import ExpertPageStreamer
    E, k, H, I, T = 8, 2, 512, 256, 48
    host = _host_pages(E, H, I, 1)
    st = ExpertPageStreamer(host, num_pages=E, device="cuda")
    perm = [3, 0, 7, 1, 6, 2, 5, 4]               # pool page of expert e
    x, logits = _inputs(T, E, H, 2)
    st.load(experts=range(E), pages=perm)
    out = st.forward(x.cuda(), logits.cuda(), k, torch.tensor(perm, device="cuda"))
    torch.cuda.synchronize()
    assert st.status(x, E, k) == 0
    _check(out, x, logits, host, list(range(E)), k)
    # second round: new weights into the same pages
    host2 = _host_pages(E, H, I, 3)
    st.host = host2
    st.load(experts=range(E), pages=perm)
    out2 = st.forward(x.cuda(), logits.cuda(), k, torch.tensor(perm, device="cuda"))
    torch.cuda.synchronize()
    assert st.status(x, E, k) == 0
    _check(out2, x, logits, host2, list(range(E)), k)


def test_page_never_ready_times_out_and_recovers():
    from ae_b200.streaming import ExpertPageStreamer
    E, k, H, I, T = 4, 2, 256, 128, 16
    host = _host_pages(E, H, I, 5)
    st = ExpertPageStreamer(host, num_pages=E, device="cuda")
    x, logits = _inputs(T, E, H, 6)
    st.load(experts=range(E))                        # epoch 1 for every page
    torch.cuda.synchronize()
    # ask for epoch 2, which nothing raises: the FFN kernel's page wait runs out (2 s)
    st.forward(x.cuda(), logits.cuda(), k, torch.arange(E, device="cuda"), epoch=st.epoch + 1)
    torch.cuda.synchronize()
    assert st.status(x, E, k) == -9  # SMB_ERR_DEVICE_TIMEOUT
    # the context is still usable: a normal round works
    st.load(experts=range(E))
    out = st.forward(x.cuda(), logits.cuda(), k, torch.arange(E, device="cuda"))
    torch.cuda.synchronize()
    assert st.status(x, E, k) == 0
    _check(out, x, logits, host, list(range(E)), k)
