"""kllm_tt_gemm, the many-row TT-GEMM (prefill shape), on the GPU.

Bar: every row bit-identical to the TT-GEMV of that row -- to the oracle's
restatement of the reference order on the shapes it finishes quickly, and to
the device TT-GEMV entry point (kllm_tt_gemv) on a prefill-sized case.
Shapes cover one chunk (K < 128), K % T != 0, N not a multiple of the
128-column tile, rows not a multiple of the 64-row tile, and 65536 codes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.device("cuda", 0))


def _device_inputs(x, cb, idx):
    return _dev(x), _dev(np.pad(cb, (0, (-len(cb)) % 4))), _dev(idx.view(np.int16))


def _gemm(dx, dc, di, codes):
    import torch

    import kmap_b200
    rows, K = dx.shape
    N = di.shape[1]
    dy = torch.full((rows, N), float("nan"), device=dx.device)
    rc = kmap_b200.lib().kllm_tt_gemm(dx.data_ptr(), rows, dc.data_ptr(), codes,
                                      di.data_ptr(), K, N, dy.data_ptr(), None)
    assert rc == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("rows,K,N,codes", [
    (1, 1024, 100, 4096), (3, 127, 9, 300), (37, 1025, 257, 5461), (64, 2048, 128, 4096),
    (130, 777, 300, 65536), (70, 5632, 130, 5461)])
def test_tt_gemm_matches_oracle_bitexact(gpu, oracle, rows, K, N, codes):
    from kmap_b200 import chipgen
    x, cb, idx = chipgen.tt_case(rows * 7 + K, K, N, codes, rows=rows)
    y = _gemm(*_device_inputs(x, cb, idx), codes)
    y_o = oracle.tt_gemv(x, cb, idx)
    assert np.array_equal(y.view(np.uint32), y_o.view(np.uint32))


def test_tt_gemm_matches_device_tt_gemv_prefill_shape(gpu):
    import torch

    import kmap_b200
    from kmap_b200 import chipgen
    rows, K, N, codes = 512, 2048, 2560, 4494
    x, cb, idx = chipgen.tt_case(5, K, N, codes, rows=rows)
    dx, dc, di = _device_inputs(x, cb, idx)
    y = _gemm(dx, dc, di, codes)
    dy = torch.empty((rows, N), device=dx.device)
    assert kmap_b200.lib().kllm_tt_gemv(dx.data_ptr(), rows, dc.data_ptr(), codes, di.data_ptr(),
                                        K, N, dy.data_ptr(), None) == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(y.view(np.uint32), dy.cpu().numpy().view(np.uint32))


def test_tt_gemm_rejects_bad_arguments(gpu):
    import kmap_b200
    lib = kmap_b200.lib()
    assert lib.kllm_tt_gemm(None, 4, None, 16, None, 8, 8, None, None) != 0
    assert "invalid arguments" in (kmap_b200.last_error() or "")
    lib.kllm_clear_error()
