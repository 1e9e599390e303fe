"""The bounded mbarrier wait of the tcgen05 kernels (GEMM, attention, DACVAE
convolution) runs out cleanly.

A probe kernel built in each kernel file waits, with that file's own
mbar_wait, on a barrier nothing ever arrives on (no GPU fault, no trap: the
wait simply never completes), with the limit shortened from 4 s to 50 ms.  The
first wait must give up after the limit and set the file's watchdog flag;
every later wait must then return at once, so a stalled launch ends after one
limit, not one per wait.  The host must see the flag (the same read the engine
turns into IRT_E_CUDA "device watchdog"), the flag must clear on read, and the
device must stay usable: a tcgen05 GEMM right after is still correct.  The
error model follows src/error.rs:3-60 (a failure is reported as an error
value, never a hang).
"""

import ctypes

import pytest

from test_gpu_kernels import check, dev, hooks, ptr  # noqa: F401  (fixture)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000
WAITS = 8


def probe_lib():
    L = hooks()
    L.irtt_watchdog_probe.argtypes = [ctypes.c_int, ctypes.c_ulonglong, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_ulonglong)]
    L.irtt_watchdog_read_and_clear.argtypes = [ctypes.c_int]
    return L


@pytest.mark.parametrize("which,name", [(0, "gemm"), (1, "attention"), (2, "conv")])
def test_bounded_wait_expires_reports_and_clears(dev, which, name):  # noqa: F811
    L = probe_lib()
    torch.cuda.synchronize()
    assert L.irtt_watchdog_read_and_clear(which) == 0, f"{name}: flag set before the probe"
    el = ctypes.c_ulonglong(0)
    rc = L.irtt_watchdog_probe(which, LIMIT_NS, WAITS, ctypes.byref(el))
    assert rc == 0, L.irtt_last_error().decode()
    ms = el.value / 1e6
    print(f"{name}: {WAITS} waits on a barrier nothing arrives on ended after {ms:.1f} ms "
          f"(limit {LIMIT_NS / 1e6:.0f} ms)")
    # one full limit for the first wait, the other waits give up at once
    assert LIMIT_NS <= el.value < 2 * LIMIT_NS, ms
    if which == 0:
        # the GEMM flag is the one irtt_sync_check (and Engine::sample) reads
        assert L.irtt_sync_check() == 20
        assert "watchdog" in L.irtt_last_error().decode()
        assert L.irtt_sync_check() == 0  # cleared on read
    else:
        assert L.irtt_watchdog_read_and_clear(which) == 1
        assert L.irtt_watchdog_read_and_clear(which) == 0
    # the device is still usable and the 4 s default limit is back
    M, N, K = 256, 256, 512
    g = torch.Generator(device="cuda").manual_seed(which)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    c = torch.empty(M, N, device="cuda")
    check(L.irtt_gemm_store(ptr(a), ptr(b), M, N, K, ptr(c), 0))
    ref = a.float() @ b.float().T
    assert ((c - ref).norm() / ref.norm()).item() < 1e-5
