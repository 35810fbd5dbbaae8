"""Data-parallel gradient sync (bucketed AllReduce with fused 1/world, small tensors as one group)
on CPU ranks over the host-memory communicator, against gradients averaged locally."""
import pytest

from tests import _mp, dp_cases

torch = pytest.importorskip("torch")


def test_bucket_layout_reverse_order_and_views():
    from originccl_b200.parallel.data_parallel import GradBuckets
    shapes = [("a", (10, 10)), ("bias", (4,)), ("b", (30,)), ("c", (7, 3))]
    gb = GradBuckets(shapes, dtype=torch.float32, bucket_bytes=64 * 4, small_bytes=16)
    # large tensors are laid out last-first: c, b, a
    assert gb.large_idx == [3, 2, 0]
    assert gb.offsets[3] == 0 and gb.offsets[2] == 21 and gb.offsets[0] == 51
    assert gb.small_idx == [1]
    assert gb.flat.numel() == 151 and gb.num_buckets == 3
    assert list(gb.buckets_of(0)) == [0, 1, 2]  # a spans [51, 151)
    gb.views[0].fill_(1.0)
    assert gb.flat[51:151].eq(1.0).all() and gb.flat[:51].eq(0.0).all()
    assert sum(gb.bucket(i).numel() for i in range(gb.num_buckets)) == gb.flat.numel()


@pytest.mark.parametrize("mode", ["sync", "attach"])
def test_dp_sync_two_ranks_matches_local_average(mode):
    res = _mp.run(2, dp_cases.run_dp_sync, mode, 16 << 10, timeout=240)
    assert res[0]["buckets"] > 1 and res[0]["small"] > 0


def test_dp_sync_three_ranks_one_bucket_per_tensor():
    res = _mp.run(3, dp_cases.run_dp_sync, "attach", 4096, timeout=240)
    assert res[0]["buckets"] > 10
