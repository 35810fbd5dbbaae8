"""The allocation-free entry point against the regular one (GPU).

bcclLocalAllReduceNoAlloc serves callers that cannot allocate device memory (a framework
allocator that owns all of it, a thread that must stay out of the driver's allocation path):
its scratch lives in a fixed device array inside the library. This test calls it through its
exported C symbol and checks, on two calls in a row (the array keeps the first call's contents),
that it matches a one-rank device communicator's AllReduce, the regular entry point, within the
tolerances the other GPU tests use. The file name makes pytest collect it last.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from tests import gpu_cases  # noqa: E402

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")


def _no_alloc_fn():
    from originccl_b200 import _native
    fn = _native.lib().bcclLocalAllReduceNoAlloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_size_t),
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    return fn


def _call(fn, srcs, dsts, dtype_code, op, scale, stream):
    n = len(srcs)
    src_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in srcs])
    dst_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in dsts])
    cnt_arr = (ctypes.c_size_t * n)(*[t.numel() for t in srcs])
    return fn(src_arr, dst_arr, cnt_arr, n, dtype_code, op, ctypes.c_float(scale), ctypes.c_void_p(stream))


@pytest.mark.parametrize("dtype,code", [("float32", 0), ("bfloat16", 4)])
def test_no_alloc_matches_regular_entry_point(dtype, code):
    _need_gpu()
    import originccl_b200 as occl
    from originccl_b200 import ReduceOp

    torch.cuda.set_device(0)
    fn = _no_alloc_fn()
    comm = occl.Communicator().init(0, 1, None, device=0, blocking=True)
    stream = torch.cuda.current_stream().cuda_stream
    td = getattr(torch, dtype)
    sizes = [1, 33, 4096, 70001, (1 << 20) + 5]
    for call, (op, scale) in enumerate([(ReduceOp.SUM, 0.5), (ReduceOp.AVG, 2.0)]):
        srcs = [gpu_cases.rank_input(0, n, dtype, seed=100 * call + i).cuda() for i, n in enumerate(sizes)]
        outs = [torch.full_like(s, 123) for s in srcs]
        assert _call(fn, srcs, outs, code, int(op), scale, stream) == 0, occl.comm._native.last_error()
        torch.cuda.synchronize()
        for i, (s, o) in enumerate(zip(srcs, outs)):
            ref = torch.empty_like(s)
            comm.all_reduce(s, op, out=ref, scale=scale)
            gpu_cases._close(o, ref, dtype, f"no-alloc call {call} tensor {i}")
    comm.destroy()


def test_no_alloc_rejects_oversized_batch():
    _need_gpu()
    torch.cuda.set_device(0)
    fn = _no_alloc_fn()
    x = torch.ones(4, device="cuda")
    too_many = 1025  # BCCL_NOALLOC_MAX_ITEMS + 1
    rc = _call(fn, [x] * too_many, [x] * too_many, 0, 0, 1.0, torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    from originccl_b200 import _native
    assert "at most 1024" in _native.last_error()
