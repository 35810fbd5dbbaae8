"""The torch.distributed "bccl" backend on CPU ranks: every supported collective through the
torch API, and DistributedDataParallel training on it, against local references."""
import pytest

from tests import _mp, torch_backend_cases

pytest.importorskip("torch")


@pytest.mark.parametrize("world", [2, 3])
def test_torch_collectives_on_bccl_backend(world):
    res = _mp.run(world, torch_backend_cases.run_collectives, timeout=240)
    assert all(r["alltoall_rejected"] for r in res)


def test_ddp_on_bccl_backend():
    res = _mp.run(2, torch_backend_cases.run_ddp, timeout=240)
    assert all(r["worst"] < 1e-6 for r in res)
