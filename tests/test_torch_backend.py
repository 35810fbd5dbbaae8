"""The torch.distributed "bccl" backend on CPU ranks: every supported collective through the
torch API, and DistributedDataParallel training on it, against local references."""
import pytest

from tests import _mp, torch_backend_cases

pytest.importorskip("torch")


@pytest.mark.parametrize("world", [2, 3])
def test_torch_collectives_on_bccl_backend(world):
    res = _mp.run(world, torch_backend_cases.run_collectives, timeout=240)
    assert all(r["bad_splits_rejected"] for r in res)


@pytest.mark.parametrize("hook", [False, True])
def test_ddp_on_bccl_backend(hook):
    res = _mp.run(2, torch_backend_cases.run_ddp, hook, timeout=240)
    assert all(r["worst"] < 1e-6 for r in res)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_ddp_cuda_on_bccl_backend():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    for hook in (False, True):
        res = _mp.run(2, torch_backend_cases.run_ddp_cuda, hook, timeout=300)
        assert all(r["worst"] < 1e-4 for r in res)


def test_subgroups_on_bccl_backend():
    res = _mp.run(4, torch_backend_cases.run_subgroups, timeout=240)
    assert [r["members"] for r in res] == [[0, 1], [0, 1], [2, 3], [2, 3]]
