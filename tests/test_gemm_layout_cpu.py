"""Host-side checks of the GEMM weight layout (no GPU): the pre-tiled layout round-trips and puts every
128 x 64 tile in one contiguous block; packing a layer keeps its CPU forward unchanged."""
import torch

from sglang_neuron_b200.ops.gemm import TiledWeight, linear


def test_tiled_weight_round_trip_and_tile_contiguity():
    torch.manual_seed(0)
    for F, K in [(128, 64), (300, 200), (5120, 2880), (1, 8)]:
        w = torch.randn(F, K)
        t = TiledWeight(w)
        ntf, nk = (F + 127) // 128, (K + 63) // 64
        assert t.data.shape == (ntf * nk * 128, 64)
        assert torch.equal(t.untiled(), w)
        # tile (f, k) is rows [(f * nk + k) * 128, +128) of the tiled buffer
        f, k = ntf - 1, nk - 1
        blk = t.data[(f * nk + k) * 128:(f * nk + k + 1) * 128]
        ref = torch.zeros(128, 64)
        sub = w[f * 128:(f + 1) * 128, k * 64:(k + 1) * 64]
        ref[: sub.shape[0], : sub.shape[1]] = sub
        assert torch.equal(blk, ref)


def test_linear_accepts_tiled_weight_on_cpu():
    torch.manual_seed(1)
    x, w, b = torch.randn(5, 200), torch.randn(300, 200), torch.randn(300)
    assert torch.allclose(linear(x, TiledWeight(w), b), torch.nn.functional.linear(x, w, b), atol=1e-4)
