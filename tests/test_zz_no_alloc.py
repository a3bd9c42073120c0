"""kllm_tt_gemv_noalloc, the allocation-free TT-GEMV entry point (GPU).

It exists for callers that must not allocate device memory (code running
under CUDA graph capture, plugins whose host owns the device memory pool,
fixed-footprint hosts), so its scratch lives in a fixed array in the
library's device image.  Checked here through the C ABI against the
allocating entry point kllm_tt_gemv, bit for bit (the TT-GEMV tolerance of
this suite), on two calls in a row, and for its column limit.  The file is
named to be collected last; it passes alone or after the other tests."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P = C.c_void_p


def _entry_points():
    import kmap_b200
    lib = kmap_b200.lib()
    f = lib.kllm_tt_gemv_noalloc
    f.restype = C.c_int
    f.argtypes = [P, P, C.c_int, P, C.c_int, C.c_int, P, P]
    return lib, f


def _device_case(K, N, codes, seed):
    import torch

    from kmap_b200 import chipgen
    x, cb, idx = chipgen.tt_case(seed, K, N, codes)
    dev = torch.device("cuda", 0)
    return (torch.from_numpy(x[0]).to(dev),
            torch.from_numpy(np.pad(cb, (0, (-len(cb)) % 4))).to(dev),
            torch.from_numpy(idx.view(np.int16)).to(dev))


@pytest.mark.parametrize("K,N,codes", [(2048, 2048, 4096), (5632, 2048, 5461), (1000, 37, 400)])
def test_noalloc_equals_allocating_entry_point_twice(K, N, codes):
    import torch

    import kmap_b200
    lib, noalloc = _entry_points()
    dev = torch.device("cuda", 0)
    for call, seed in enumerate((11, 12)):          # two calls in a row
        x, cb, idx = _device_case(K, N, codes, seed)
        y_ref = torch.empty(N, device=dev)
        y_na = torch.full((N,), float("nan"), device=dev)
        assert lib.kllm_tt_gemv(x.data_ptr(), 1, cb.data_ptr(), codes, idx.data_ptr(), K, N,
                                y_ref.data_ptr(), None) == 0, kmap_b200.last_error()
        assert noalloc(x.data_ptr(), cb.data_ptr(), codes, idx.data_ptr(), K, N,
                       y_na.data_ptr(), None) == 0, kmap_b200.last_error()
        torch.cuda.synchronize()
        a = y_ref.cpu().numpy().view(np.uint32)
        b = y_na.cpu().numpy().view(np.uint32)
        assert np.array_equal(a, b), (K, N, call)


def test_noalloc_rejects_more_columns_than_its_scratch():
    import kmap_b200
    lib, noalloc = _entry_points()
    buf = (C.c_float * 16)()
    rc = noalloc(C.addressof(buf), C.addressof(buf), 4, C.addressof(buf), 8, 65537,
                 C.addressof(buf), None)
    assert rc != 0
    assert "65536" in (kmap_b200.last_error() or "")
    lib.kllm_clear_error()


def test_noalloc_leaves_device_memory_untouched():
    """After one warm-up call (which looks up the scratch array's address),
    further calls change neither the device's free memory nor what torch's
    allocator holds: the entry point allocates nothing."""
    import torch

    import kmap_b200
    lib, noalloc = _entry_points()
    K, N, codes = 2048, 2048, 4096
    x, cb, idx = _device_case(K, N, codes, 21)
    y = torch.empty(N, device="cuda")
    call = lambda: noalloc(x.data_ptr(), cb.data_ptr(), codes, idx.data_ptr(), K, N,
                           y.data_ptr(), None)
    assert call() == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    held0 = torch.cuda.memory_reserved()
    for _ in range(5):
        assert call() == 0, kmap_b200.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0 and torch.cuda.memory_reserved() == held0
