"""tcgen05 GEMM numerics against an fp32 PyTorch reference (GPU)."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _need():
    from originccl_b200.ops import gemm
    if not gemm.available():
        pytest.skip("needs an sm_100 GPU")
    return gemm


@pytest.mark.parametrize("kernel", ["1", "0"], ids=["pair_256x256", "single_128x256"])
@pytest.mark.parametrize("m,n,k,act", [
    (128, 256, 64, None),        # one tile, one k-block
    (256, 512, 1024, None),      # several tiles and k-blocks
    (300, 200, 136, "silu"),     # ragged M, N and K (TMA zero fill + masked stores)
    (1024, 3584, 2048, "silu"),  # TP up-projection shape (scaled down in K)
    (384, 256, 64, None),        # an odd number of 2-SM row blocks (the last pair half-empty)
])
def test_gemm_matches_fp32_reference(m, n, k, act, kernel, monkeypatch):
    gemm = _need()
    monkeypatch.setenv("BCCL_GEMM_PAIR", kernel)
    assert gemm.kernel_name() == ("pair_256x256" if kernel == "1" else "single_128x256")
    torch.manual_seed(0)
    a = (torch.randn(m, k, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    y = gemm.gemm(a, w, act)
    assert gemm.check_error() == 0
    ref = a.float() @ w.float().t()
    if act == "silu":
        ref = torch.nn.functional.silu(ref)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())


@pytest.mark.parametrize("m,n,k,act", [
    (256, 224, 64, None),        # one tile
    (300, 200, 136, "silu"),     # ragged in every dimension
    (1024, 3584, 2048, "silu"),  # 16 full column tiles
    (512, 1000, 320, None),      # a partial last column tile
])
def test_gemm_224_wide_tiles_match_fp32_reference(m, n, k, act, monkeypatch):
    gemm = _need()
    monkeypatch.setenv("BCCL_GEMM_PAIR", "1")
    monkeypatch.setenv("BCCL_GEMM_BN", "224")
    torch.manual_seed(1)
    a = (torch.randn(m, k, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    y = gemm.gemm(a, w, act)
    assert gemm.check_error() == 0
    ref = a.float() @ w.float().t()
    if act == "silu":
        ref = torch.nn.functional.silu(ref)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
