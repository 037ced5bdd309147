"""Failure detection on the device, without faulting or hanging the GPU.

Every mbarrier wait in the kernels is bounded (2 s of %globaltimer); when one gives up,
the kernel sets a device error word, drains the copies and MMAs it has in flight, frees
its tensor memory and exits.  ``ee_debug_drop_next_gemm_load`` makes exactly that
happen: the next single-CTA gated GEMM's CTA 0 never issues the copies (nor the barrier
arrival) of its first K stage, so its MMA warp's wait runs out.  The test checks that
the call returns, that ``device_check`` reports the error word, and that the next call
through the same router -- which re-zeroes its workspace header by itself after the
reported error -- is bit-identical to a clean run.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(M, n, K, N, device):
    g = torch.Generator().manual_seed(31)
    s = torch.exp(torch.rand(M, 1, generator=g) * 2.0 + 1.0)
    logits = (torch.randn(M, n, generator=g) * s).half().to(device)
    a = torch.randn(M, K, generator=g).half().to(device)
    w = (torch.randn(N, K, generator=g) * 0.02).half().to(device)
    return logits, a, w


def test_gemm_wait_timeout_is_reported_and_the_next_call_is_clean(pkg, cuda):
    lib = pkg.load_library()
    M, n, K, N = 512, 1024, 4096, 4096
    logits, a, w = _inputs(M, n, K, N, cuda)
    pack = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    r = pkg.EntropyRouter(0.41, 1.68, k_split=False)
    r.reserve(M, K, cuda)
    assert lib.ee_set_gemm_policy(1) == 0  # the single-CTA kernel, where the hook acts
    try:
        r.route(logits)
        y_ref = r.gated_linear(a, pack)
        torch.cuda.synchronize()
        assert pkg._lib.device_check() == 0
        counts = r.counts.cpu().tolist()
        assert sum(counts) == M and min(counts) > 0  # all three buckets take part

        assert lib.ee_debug_drop_next_gemm_load(0) == 0
        r.route(logits)
        t0 = time.perf_counter()
        y_bad = r.gated_linear(a, pack)
        torch.cuda.synchronize()  # returns: the wait gave up, the CTA unwound
        elapsed = time.perf_counter() - t0
        with pytest.raises(RuntimeError, match=r"EE_ERR_DEVICE.*word 0x1 "):
            pkg._lib.device_check()
        assert 1.5 < elapsed < 30.0, elapsed  # the 2 s wait limit, not a hang
        assert pkg._lib.device_check() == 0  # reading the word cleared it
        assert not torch.equal(y_bad, y_ref)  # CTA 0's tile was never written

        # the same router again: header re-zeroed by itself, results bit-identical
        for _ in range(2):
            r.route(logits)
            y = r.gated_linear(a, pack)
            torch.cuda.synchronize()
            assert pkg._lib.device_check() == 0
            assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
            assert r.counts.cpu().tolist() == counts
    finally:
        lib.ee_set_gemm_policy(0)


def test_drop_hook_rejects_a_cta_outside_the_grid(pkg, cuda):
    lib = pkg.load_library()
    assert lib.ee_debug_drop_next_gemm_load(-1) == -1
    assert lib.ee_debug_drop_next_gemm_load(100000) == -1
