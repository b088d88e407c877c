"""Host-side logic of the pair conditioning: the weight copy that ``tmu_pair_cond`` reads
(``PairCondWeights.from_head``) holds exactly the matrices the oracle restates from
``diffusion_params`` (mlx_diffusion.py:85-92, pair16 casts mlx_diffusion16.py:224-227)."""

from __future__ import annotations

import torch

from esmfold2_mlx_b200.pair_cond import PairCondWeights
from esmfold2_mlx_b200.synthetic import DiffusionHead
from oracle import pair_cond_oracle as pco


def test_weight_copy_matches_the_reference_folding():
    head = DiffusionHead(128, 128, 128, 256, 2, 3, 8, seed=4)
    w = PairCondWeights.from_head(head, "cpu")
    p = pco.pair_cond_params(head)
    t = w.tensors
    assert (w.c_in, w.c_pair, w.hidden, w.heads, w.n_bias) == (256, 128, 256, 8, 24)
    assert torch.equal(t["proj"].float().T, p["proj"])
    assert torch.equal(t["bias_w"].float().T, p["bias_w"])
    assert torch.equal(t["bias_b"].float(), p["bias_b"])
    assert torch.equal(t["ln_w"], p["ln_w"]) and torch.equal(t["ln_b"], p["ln_b"])
    for tw, tp in zip(t["transitions"], p["transitions"]):
        a, b = tw["w12"].float().chunk(2, 0)
        assert torch.equal(a.T, tp["a"]) and torch.equal(b.T, tp["b"])
        assert torch.equal(tw["w3"].float().T, tp["out"])
        assert torch.equal(tw["ln_w"], tp["ln_w"])


def test_oracle_layout_is_blocks_batch_heads_rows_cols():
    """out[k, b, h, i, j] = bias[b, i, j, k * H + h] (mlx_diffusion.py:259)."""
    head = DiffusionHead(128, 128, 128, 256, 1, 2, 8, seed=1)
    p = pco.pair_cond_params(head)
    zt, rp = torch.randn(2, 5, 5, 128), torch.randn(2, 5, 5, 128)
    out = pco.pair_biases_fp16(p, zt, rp)
    assert out.shape == (2, 2, 8, 5, 5)
    # recompute one channel by hand from the flat form
    x = torch.cat([zt, rp], -1)
    z = pco.r16(pco.r16(pco.layer_norm(x, p["ln_w"], p["ln_b"], 1e-5)) @ p["proj"])
    for tr in p["transitions"]:
        hh = pco.r16(pco.layer_norm(z, tr["ln_w"], tr["ln_b"], 1e-5))
        xa, xb = pco.r16(hh @ tr["a"]), pco.r16(hh @ tr["b"])
        z = z + pco.r16(pco.r16(pco.r16(xa * pco.r16(pco.sigmoid(xa))) * xb) @ tr["out"])
    flat = pco.r16(pco.r16(pco.r16(pco.layer_norm(z, torch.ones(128), torch.zeros(128), 1e-5)) @ p["bias_w"])
                   + p["bias_b"])
    assert torch.equal(out[1, 0, 3], flat[0, :, :, 1 * 8 + 3])
