"""The tensor-core prefill TT-GEMM (kllm_tt_gemm_tc, tcgen05 + TMEM + TMA).

Codebooks of bf16 numbers (the compiler's codebooks of bf16 checkpoints),
x ~ N(0, 1) fp32 split into 2 or 3 bf16 terms.  Checked against the exact
product computed in float64 on the host and against the bit-exact FP32
TT-GEMM (kllm_tt_gemm): with 3 terms the error is the tensor core's fp32
accumulation (a few 1e-6 of the row's sum of |x w|); with 2 terms x itself
is carried to 2^-17.  Shapes: one and several 128-row tiles,
ragged row counts (the tensor map fills rows past the end with zeros and the
epilogue skips them), N multiples of 128 and 256, K = 64 .. 14336; up to
64 rows (decode of several sequences) through the split-K form."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bf16_codebook(rng, n):
    v = (rng.standard_normal(4 * n) * 0.02).astype(np.float32)
    v = (v.view(np.uint32) & np.uint32(0xffff0000)).view(np.float32)
    return np.unique(v)[:n]


def _case(seed, R, K, N, codes=4096):
    rng = np.random.default_rng(seed)
    cb = _bf16_codebook(rng, codes)
    idx = rng.integers(0, len(cb), (K, N)).astype(np.uint16)
    x = rng.standard_normal((R, K)).astype(np.float32)
    return x, cb, idx


def _run(fn, x, cb, idx, *extra):
    import torch

    import kmap_b200
    dev = torch.device("cuda", 0)
    R, K = x.shape
    N = idx.shape[1]
    dx = torch.from_numpy(x).to(dev)
    dc = torch.from_numpy(np.pad(cb, (0, (-len(cb)) % 4))).to(dev)
    di = torch.from_numpy(idx.view(np.int16)).to(dev)
    dy = torch.full((R, N), float("nan"), device=dev)
    s = torch.cuda.current_stream()
    rc = fn(dx.data_ptr(), R, dc.data_ptr(), len(cb), di.data_ptr(), K, N, dy.data_ptr(),
            *extra, s.cuda_stream)
    assert rc == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("R,K,N", [(128, 64, 128), (128, 2048, 256), (200, 1024, 384),
                                   (1, 2048, 2048), (300, 5632, 256), (513, 2048, 2560),
                                   # few rows (<= 64): the weight on the MMA's 128-row
                                   # side, K split over ranges summed in order
                                   (32, 4096, 6144), (17, 14336, 4096), (64, 4096, 28672),
                                   (5, 1024, 128), (33, 256, 640)])
@pytest.mark.parametrize("terms", [3, 2])
def test_tc_gemm_against_float64(gpu, R, K, N, terms):
    import kmap_b200
    lib = kmap_b200.lib()
    x, cb, idx = _case(R * 7 + K + N, R, K, N)
    w = cb[idx].astype(np.float64)
    exact = x.astype(np.float64) @ w
    scale = np.abs(x).astype(np.float64) @ np.abs(w)   # sum of |x w| per output
    y = _run(lib.kllm_tt_gemm_tc, x, cb, idx, terms)
    assert np.isfinite(y).all()
    y_ref_order = _run(lib.kllm_tt_gemm, x, cb, idx)   # the reference's fp32 order
    err = (np.abs(y - exact) / np.maximum(scale, 1e-30)).max()
    err_ref = (np.abs(y_ref_order - exact) / np.maximum(scale, 1e-30)).max()
    # 3 terms: x is carried whole and every product is exact; what remains
    # is the tensor core's fp32 accumulation, which aligns each K-step's
    # products before adding them (measured ~1-2.3e-6 of sum |x w|, ~20x the
    # serial fp32 order's error err_ref); 2 terms: x itself carried to 2^-17
    bound = 5e-6 if terms == 3 else 2e-5
    assert err < bound, (err, err_ref)
    np.testing.assert_allclose(y, y_ref_order, rtol=1e-4, atol=1e-4 * np.abs(exact).max())


def test_tc_gemm_rejects_non_bf16_codebook(gpu):
    import kmap_b200
    lib = kmap_b200.lib()
    x, cb, idx = _case(1, 128, 128, 128)
    cb = cb.copy()
    cb[3] = np.float32(0.0123456)
    with pytest.raises(AssertionError):
        _run(lib.kllm_tt_gemm_tc, x, cb, idx, 3)
    assert "bf16" in (kmap_b200.last_error() or "")
    lib.kllm_clear_error()
