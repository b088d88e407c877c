"""Seeded synthetic trunks and pair tensors with the shapes the reference's benchmarks use.

Biohub's checkpoints and the ``esm`` package are not available here, so benchmarks and tests
build a module tree with the attribute names the reference reads when it copies a trunk's
weights (``src/esmfold2_mlx/mlx_trunk.py:40-67``; ``fast_trunk.py:52-56``):

    folding_trunk.blocks[i].tri_mul_out._engine.{latent_channels, norm_start, proj_bundle,
                                                norm_mix, proj_emit, proj_gate}
    folding_trunk.blocks[i].tri_mul_in._engine.{...}
    folding_trunk.blocks[i].pair_transition.{norm, ffn.w12, ffn.w3, ffn.hidden_features}

Weights are N(0, 1/fan_in); LayerNorm gamma=1, beta=0 unless ``ln_noise`` is set; Linear
layers have no bias, as in the reference (``fast_trunk.py:53,59``).  Optional tri-mul biases
(N(0, 0.02), one benchmark configuration adds them) are returned separately because the
reference module tree has no place for them.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn


def _linear(out_f: int, in_f: int, g: torch.Generator) -> nn.Linear:
    lin = nn.Linear(in_f, out_f, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(out_f, in_f, generator=g) / in_f**0.5)
    return lin


def _ln(ch: int, g: torch.Generator, noise: float) -> nn.LayerNorm:
    ln = nn.LayerNorm(ch)
    if noise:
        with torch.no_grad():
            ln.weight.copy_(1.0 + noise * torch.randn(ch, generator=g))
            ln.bias.copy_(noise * torch.randn(ch, generator=g))
    return ln


class TriangleMultiplicativeBlock(nn.Module):
    """Holds the weights of one triangle update under the names the reference reads."""

    def __init__(self, c_z: int, c: int, g: torch.Generator, ln_noise: float = 0.0):
        super().__init__()
        self.latent_channels = c
        self.norm_start = _ln(c_z, g, ln_noise)
        self.proj_bundle = _linear(4 * c, c_z, g)  # rows [signal_a | signal_b | gate_a | gate_b]
        self.norm_mix = _ln(c, g, ln_noise)
        self.proj_emit = _linear(c_z, c, g)
        self.proj_gate = _linear(c_z, c_z, g)


class TriangleMultiplicativeUpdate(nn.Module):
    def __init__(self, c_z: int, c: int, g: torch.Generator, ln_noise: float = 0.0):
        super().__init__()
        self._engine = TriangleMultiplicativeBlock(c_z, c, g, ln_noise)


class _FFN(nn.Module):
    def __init__(self, c_z: int, hidden: int, g: torch.Generator, activation: str):
        super().__init__()
        self.hidden_features = hidden
        self.activation = activation
        width = 2 * hidden if activation == "swiglu" else hidden
        self.w12 = _linear(width, c_z, g)
        self.w3 = _linear(c_z, hidden, g)


class Transition(nn.Module):
    def __init__(self, c_z: int, hidden: int, g: torch.Generator, activation: str = "swiglu",
                 ln_noise: float = 0.0):
        super().__init__()
        self.norm = _ln(c_z, g, ln_noise)
        self.ffn = _FFN(c_z, hidden, g, activation)


class PairUpdateBlock(nn.Module):
    def __init__(self, c_z: int, c: int, hidden: int, g: torch.Generator, activation: str, ln_noise: float):
        super().__init__()
        self.tri_mul_out = TriangleMultiplicativeUpdate(c_z, c, g, ln_noise)
        self.tri_mul_in = TriangleMultiplicativeUpdate(c_z, c, g, ln_noise)
        self.pair_transition = Transition(c_z, hidden, g, activation, ln_noise)


class FoldingTrunk(nn.Module):
    """A trunk-shaped module tree; its own forward is never used (the swap replaces it)."""

    def __init__(self, n_blocks: int, c_z: int = 128, c: int = 128, hidden: int | None = None,
                 seed: int = 0, activation: str = "swiglu", ln_noise: float = 0.0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        hidden = hidden if hidden is not None else 4 * c_z
        self.blocks = nn.ModuleList(
            PairUpdateBlock(c_z, c, hidden, g, activation, ln_noise) for _ in range(n_blocks))
        self.chunk_size = None
        self.kernel_backend = None

    def set_chunk_size(self, chunk_size):
        self.chunk_size = chunk_size

    def set_kernel_backend(self, backend):
        self.kernel_backend = backend


class FoldModel(nn.Module):
    """Minimal model object with a ``folding_trunk`` attribute, for the variant registry."""

    def __init__(self, folding_trunk: nn.Module):
        super().__init__()
        self.folding_trunk = folding_trunk


class _TransitionLayer(nn.Module):
    """``TransitionLayer``: LN -> silu(h @ a) * (h @ b) -> out (``mlx_diffusion.py:51-52``)."""

    def __init__(self, c: int, hidden: int, g: torch.Generator, ln_noise: float):
        super().__init__()
        self.norm = _ln(c, g, ln_noise)
        self.a_proj = _linear(hidden, c, g)
        self.b_proj = _linear(hidden, c, g)
        self.out_proj = _linear(c, hidden, g)


class _AttnPairBias(nn.Module):
    """The pair-bias part of one token-transformer attention block (``mlx_diffusion.py:87-89``)."""

    def __init__(self, c: int, heads: int, g: torch.Generator, ln_noise: float):
        super().__init__()
        self.num_heads = heads
        self.pair_norm = _ln(c, g, ln_noise)
        self.pair_bias_proj = _linear(heads, c, g)


class DiffusionHead(nn.Module):
    """The diffusion head's pair-conditioning weights under the names the reference reads
    (``mlx_diffusion.py:61-64,85-92``): ``diffusion_module.conditioning.{z_input_norm, z_proj,
    z_transitions[k].{norm, a_proj, b_proj, out_proj}}`` and
    ``diffusion_module.token_transformer.attn_blocks[i].{pair_norm, pair_bias_proj, num_heads}``.
    The checkpoint's sizes are not public here; the defaults take c_trunk = c_rel = 256 (the
    reference's "[L, L, 512]" concat, ``mlx_diffusion.py:322``), c_pair = 256, two transitions of
    width 2 c_pair and 12 blocks x 16 heads (its "12 token-attention pair biases", ``:5``)."""

    def __init__(self, c_trunk: int = 256, c_rel: int = 256, c_pair: int = 256, hidden: int = 512,
                 n_transitions: int = 2, n_blocks: int = 12, heads: int = 16, seed: int = 0,
                 ln_noise: float = 0.1):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        cond = nn.Module()
        cond.z_input_norm = _ln(c_trunk + c_rel, g, ln_noise)
        cond.z_proj = _linear(c_pair, c_trunk + c_rel, g)
        cond.z_transitions = nn.ModuleList(_TransitionLayer(c_pair, hidden, g, ln_noise) for _ in range(n_transitions))
        tt = nn.Module()
        tt.attn_blocks = nn.ModuleList(_AttnPairBias(c_pair, heads, g, ln_noise) for _ in range(n_blocks))
        self.diffusion_module = nn.Module()
        self.diffusion_module.conditioning = cond
        self.diffusion_module.token_transformer = tt


def trimul_biases(c_z: int, c: int, seed: int, std: float = 0.02) -> dict:
    """Biases for one tri-mul: proj (4c, reference column order), emit (c_z), gate (c_z)."""
    g = torch.Generator().manual_seed(seed)
    return {
        "b_in": std * torch.randn(4 * c, generator=g),
        "b_emit": std * torch.randn(c_z, generator=g),
        "b_gate": std * torch.randn(c_z, generator=g),
    }


def pair_tensor(B: int, L: int, c_z: int, seed: int) -> torch.Tensor:
    """z ~ N(0, 1), fp32, generated on the CPU so every consumer sees identical values."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, L, L, c_z, generator=g)


def pair_mask(B: int, L: int, n_pad: int = 0) -> torch.Tensor:
    """Pair mask m_i * m_j with the last ``n_pad`` residues masked out (padding)."""
    m = torch.ones(B, L)
    if n_pad:
        m[:, L - n_pad:] = 0.0
    return m[:, :, None] * m[:, None, :]


@dataclass(frozen=True)
class Config:
    """One synthetic workload (the five benchmark configurations)."""

    name: str
    L: int
    B: int = 1
    c_z: int = 128
    c: int = 128
    seed: int = 0
    n_pad: int = 0
    biases: bool = False
    directions: tuple = ("out",)
    blocks: int = 0
    recycles: int = 0
    transition: str = "swiglu"

    @property
    def pair_cells_per_step(self) -> int:
        """L^2 x tri-mul blocks in one step (all folds)."""
        n_tm = len(self.directions) if not self.blocks else 2 * self.blocks * max(1, self.recycles)
        return self.B * self.L * self.L * n_tm


CONFIGS = {
    "c1": Config("c1_L76_out", L=76, seed=0, directions=("out",)),
    "c2": Config("c2_L238_out_in_mask_bias", L=238, seed=1, n_pad=24, biases=True, directions=("out", "in")),
    "c3": Config("c3_L384_16blk_3rec_relu", L=384, seed=2, blocks=16, recycles=3, transition="relu"),
    "c4": Config("c4_64x_L146_out_in", L=146, B=64, seed=100, directions=("out", "in")),
    "c5": Config("c5_L3072_out_in", L=3072, seed=3, directions=("out", "in")),
    "L2048": Config("L2048_out_in", L=2048, seed=4, directions=("out", "in")),
    # c_z = c = 256, the width of ESMFold2's released trunk, on config 2's and L2048's shapes
    "c2w": Config("c2w_L238_cz256_out_in_mask_bias", L=238, c_z=256, c=256, seed=1, n_pad=24, biases=True,
                  directions=("out", "in")),
    "L2048w": Config("L2048w_cz256_out_in", L=2048, c_z=256, c=256, seed=4, directions=("out", "in")),
}


@dataclass(frozen=True)
class Workload:
    """One configuration's seeded inputs, all on the CPU: the trunk-shaped module tree holding
    its tri-mul weights, the optional per-direction biases, the step's input ``z`` (fp16) and
    the pair mask (fp16, or None for an all-ones mask)."""

    cfg: Config
    trunk: FoldingTrunk
    biases: dict
    z: torch.Tensor
    mask: torch.Tensor | None


def pair_rows(L: int, c_z: int, seed: int, r0: int, r1: int, block: int = 128) -> torch.Tensor:
    """Rows [r0, r1) of one fold's z ~ N(0, 1) [1, L, L, c_z] fp32 generated in blocks of ``block``
    rows, block k from its own generator (seed * 1000 + k), so that each rank of a row-sharded
    run draws only its own rows and every rank's rows agree with the whole tensor's."""
    out = torch.empty(1, r1 - r0, L, c_z)
    for k in range(r0 // block, (r1 + block - 1) // block):
        b0, b1 = k * block, min(L, (k + 1) * block)
        g = torch.Generator().manual_seed(seed * 1000 + k)
        blk = torch.randn(1, b1 - b0, L, c_z, generator=g)
        s0, s1 = max(b0, r0), min(b1, r1)
        out[:, s0 - r0:s1 - r0] = blk[:, s0 - b0:s1 - b0]
    return out


def workload(name: str, rank: int = 0, world: int = 1) -> Workload:
    """The inputs the benchmark times for configuration ``name`` on rank ``rank`` of ``world``;
    the parity tests use exactly these.

    * ``c4`` (64 folds, strong scaling): the rank's share of the folds, fold ``idx`` drawn with
      seed 100 + idx (the configuration's per-fold seeds);
    * ``c5`` (one long fold, row-sharded): the rank's rows, drawn block by block (``pair_rows``);
    * the others: one fold group per rank, drawn with seed + rank (weak scaling)."""
    cfg = CONFIGS[name]
    trunk = FoldingTrunk(1, cfg.c_z, cfg.c, seed=cfg.seed)
    biases = {d: (trimul_biases(cfg.c_z, cfg.c, cfg.seed + 31 + i) if cfg.biases else None)
              for i, d in enumerate(("out", "in"))}
    if name == "c4":
        if cfg.B % world:
            raise ValueError(f"{cfg.B} folds do not split over {world} ranks")
        per = cfg.B // world
        z = torch.cat([pair_tensor(1, cfg.L, cfg.c_z, cfg.seed + idx) for idx in range(rank * per, (rank + 1) * per)])
        B = per
    elif name == "c5":
        Lr = cfg.L // world
        z = pair_rows(cfg.L, cfg.c_z, cfg.seed, rank * Lr, (rank + 1) * Lr)
        B = cfg.B
    else:
        z = pair_tensor(cfg.B, cfg.L, cfg.c_z, cfg.seed + rank)
        B = cfg.B
    mask = pair_mask(B, cfg.L, cfg.n_pad).half() if cfg.n_pad else None
    if name == "c5" and mask is not None:
        mask = mask[:, rank * Lr:(rank + 1) * Lr].contiguous()
    return Workload(cfg, trunk, biases, z.half(), mask)


def recycle_workload(name: str = "c3"):
    """The trunk-recycle configuration's inputs (CPU): the stack (``cfg.blocks`` blocks with the
    configuration's transition, hidden 4 c_z) and its z0 ~ N(0, 1) fp32."""
    cfg = CONFIGS[name]
    trunk = FoldingTrunk(cfg.blocks, cfg.c_z, cfg.c, hidden=4 * cfg.c_z, seed=cfg.seed, activation=cfg.transition)
    return cfg, trunk, pair_tensor(1, cfg.L, cfg.c_z, cfg.seed)
