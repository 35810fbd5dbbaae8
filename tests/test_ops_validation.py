"""Argument checks of the GEMM and fused tensor-parallel ops (CPU): wrong dtypes, shapes, output
buffers and devices are rejected in Python, before any pointer reaches a kernel."""
import types

import pytest

torch = pytest.importorskip("torch")

from originccl_b200.ops import gemm, tp  # noqa: E402

COMM = types.SimpleNamespace(world_size=2, device=0)
bf = torch.bfloat16


def test_all_gather_gemm_rejects_bad_operands():
    x, w = torch.zeros(128, 64, dtype=bf), torch.zeros(96, 64, dtype=bf)
    with pytest.raises(TypeError, match="bfloat16"):
        tp.all_gather_gemm(COMM, x.float(), w)
    with pytest.raises(ValueError, match="differ in K"):
        tp.all_gather_gemm(COMM, x, torch.zeros(96, 32, dtype=bf))
    with pytest.raises(ValueError, match="2-D"):
        tp.all_gather_gemm(COMM, x[None], w)
    with pytest.raises(ValueError, match="contiguous"):
        tp.all_gather_gemm(COMM, x, w, out=torch.zeros(128, 96, dtype=bf))  # needs [256, 96]
    with pytest.raises(ValueError, match="activation"):
        tp.all_gather_gemm(COMM, x, w, activation="gelu")
    with pytest.raises(ValueError, match="CUDA"):
        tp.all_gather_gemm(COMM, x, w)


def test_gemm_reduce_scatter_rejects_bad_operands():
    h, w = torch.zeros(256, 96, dtype=bf), torch.zeros(64, 96, dtype=bf)
    with pytest.raises(ValueError, match="split"):
        tp.gemm_reduce_scatter(COMM, torch.zeros(255, 96, dtype=bf), w)
    with pytest.raises(TypeError, match="bfloat16"):
        tp.gemm_reduce_scatter(COMM, h, w.half())
    with pytest.raises(ValueError, match="contiguous"):
        tp.gemm_reduce_scatter(COMM, h, w, out=torch.zeros(64, 128, dtype=bf).t())  # [128, 64] but strided
    with pytest.raises(ValueError, match="CUDA"):
        tp.gemm_reduce_scatter(COMM, h, w)


def test_gemm_rejects_bad_operands():
    a, w = torch.zeros(128, 64, dtype=bf), torch.zeros(96, 64, dtype=bf)
    with pytest.raises(TypeError):
        gemm.gemm(a.float(), w)
    with pytest.raises(ValueError, match="shape"):
        gemm.gemm(a, torch.zeros(96, 32, dtype=bf))
    with pytest.raises(ValueError, match="activation"):
        gemm.gemm(a, w, "relu")
    with pytest.raises(ValueError, match="CUDA"):
        gemm.gemm(a, w)


def test_collectives_reject_mismatched_buffers_before_the_library():
    """A host communicator (no GPU needed) checks sizes, dtypes and memory kind in Python."""
    import numpy as np

    import originccl_b200 as occl

    comm = occl.Communicator().init(0, 1, None)  # one rank, host memory
    try:
        x = np.arange(8, dtype=np.float32)
        with pytest.raises(ValueError, match="all_reduce"):
            comm.all_reduce(x, out=np.zeros(4, dtype=np.float32))
        with pytest.raises(ValueError, match="dtype"):
            comm.all_reduce(x, out=np.zeros(8, dtype=np.float64))
        with pytest.raises(ValueError, match="all_gather"):
            comm.all_gather(np.zeros(7, dtype=np.float32), x)
        with pytest.raises(ValueError, match="reduce_scatter"):
            comm.reduce_scatter(np.zeros(8, dtype=np.float32), np.zeros(9, dtype=np.float32))
        y = np.zeros(8, dtype=np.float32)
        comm.all_reduce(x, out=y)  # matching buffers still run
        assert np.array_equal(x, y)
        if torch.cuda.is_available():
            with pytest.raises(ValueError, match="CUDA"):
                comm.all_reduce(torch.zeros(8, device="cuda"))
    finally:
        comm.destroy()
