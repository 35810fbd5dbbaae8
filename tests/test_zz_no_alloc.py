"""The allocation-free entry point (GPU).

bcclLocalAllReduceNoAlloc serves callers that cannot allocate device memory: a framework whose
caching allocator owns every byte of the device, a latency-critical thread that must stay out of
the driver's allocation path (cudaMalloc / cudaFree can synchronise the device), a tool that must
not change the process's memory footprint. Its scratch lives in a fixed device array inside the
library. These tests call it through its exported C symbol and check, on two calls in a row (the
array keeps the first call's contents), that it matches both the regular entry point (a one-rank
device communicator's AllReduce) and an independent PyTorch reference (one rank: dst = src
times the scale for floating types, src for integers, AVG over one rank being the identity),
within the tolerances the other GPU tests use; that free device memory does not change across a
call; and that bad arguments are rejected. The file name makes pytest collect it last.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from tests import gpu_cases  # noqa: E402

pytestmark = pytest.mark.gpu

CODES = {"float32": 0, "float64": 1, "int32": 2, "int64": 3, "bfloat16": 4, "float16": 5}


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


def _call(fn, srcs, dsts, dtype_code, op, scale, stream, counts=None):
    n = len(srcs)
    src_arr = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in srcs])
    dst_arr = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in dsts])
    cnt = counts if counts is not None else [t.numel() for t in srcs]
    cnt_arr = (ctypes.c_size_t * max(n, 1))(*cnt)
    return fn(src_arr, dst_arr, cnt_arr, n, dtype_code, op, ctypes.c_float(scale), ctypes.c_void_p(stream))


def _expected(src, scale):
    """One rank: every reduction is the input itself; floating types are then scaled."""
    if src.dtype in (torch.int32, torch.int64):
        return src.clone()
    return (src.double() * scale).to(src.dtype)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "int32", "int64"])
@pytest.mark.parametrize("in_place", [False, True])
def test_no_alloc_matches_regular_entry_point_and_torch(dtype, in_place):
    _need_gpu()
    import originccl_b200 as occl
    from originccl_b200 import ReduceOp, _native

    torch.cuda.set_device(0)
    fn = _no_alloc_fn()
    comm = occl.Communicator().init(0, 1, None, device=0, blocking=True)
    stream = torch.cuda.current_stream().cuda_stream
    sizes = [1, 33, 4096, 70001, (1 << 20) + 5]
    for call, (op, scale) in enumerate([(ReduceOp.SUM, 0.5), (ReduceOp.AVG, 2.0)]):
        srcs = [gpu_cases.rank_input(0, n, dtype, seed=100 * call + i).cuda() for i, n in enumerate(sizes)]
        keep = [s.clone() for s in srcs]
        outs = srcs if in_place else [torch.full_like(s, 123) for s in srcs]
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        assert _call(fn, srcs, outs, CODES[dtype], int(op), scale, stream) == 0, _native.last_error()
        torch.cuda.synchronize()
        if call == 1:  # the first call may load the module (lazy loading); later ones add nothing
            assert torch.cuda.mem_get_info()[0] == free0, "the no-alloc call changed free device memory"
        for i, (s, o) in enumerate(zip(keep, outs)):
            what = f"no-alloc {dtype} call {call} tensor {i}{' in place' if in_place else ''}"
            gpu_cases._close(o, _expected(s, scale), dtype, what + " vs torch")
            ref = torch.empty_like(s)
            comm.all_reduce(s, op, out=ref, scale=scale)
            gpu_cases._close(o, ref, dtype, what + " vs the regular entry point")
    comm.destroy()


def test_no_alloc_rejects_bad_arguments():
    _need_gpu()
    from originccl_b200 import _native

    torch.cuda.set_device(0)
    fn = _no_alloc_fn()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.ones(4, device="cuda")
    too_many = 1025  # BCCL_NOALLOC_MAX_ITEMS + 1
    assert _call(fn, [x] * too_many, [x] * too_many, 0, 0, 1.0, stream) != 0
    assert "at most 1024" in _native.last_error()
    assert _call(fn, [x], [x], 9, 0, 1.0, stream) != 0  # no such dtype
    assert "invalid dtype" in _native.last_error()
    assert _call(fn, [x], [x], 0, 7, 1.0, stream) != 0  # no such op
    assert "invalid dtype" in _native.last_error()
    # Nothing to do succeeds and launches nothing: no tensors, or only empty ones.
    assert _call(fn, [], [], 0, 0, 1.0, stream) == 0
    y = torch.full((4,), 5.0, device="cuda")
    assert _call(fn, [x], [y], 0, 0, 1.0, stream, counts=[0]) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, torch.full((4,), 5.0, device="cuda"))
