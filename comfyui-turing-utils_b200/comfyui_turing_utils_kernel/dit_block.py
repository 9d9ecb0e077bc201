"""Wan2.1-style DiT block on this package's kernels, with Megatron tensor
parallelism over torch.distributed (dim 5120, 40 heads of
128, FFN 13824, L = 75600 video tokens, 512 text tokens).

The reference plugin supplies this block's pieces but not the block (its
forward lives in ComfyUI, absent from the reference): the ConvRot quantized
linears for q/k/v/o, cross-attention and FFN (quantization/dispatch.py,
fusions.py:45-122 folds tanh-GELU into the FFN-down quantizer), the
self-attention hand-off with row-scope RMSNorm + interleaved RoPE fused into
the INT8 Q/K quantizer (adapters/wan.py:55-137), and LayerNorm + AdaLN
(ops.py:399-418).  The block structure is the published Wan2.1 one:

    h = LN(x) * (1 + scale_msa) + shift_msa
    x = x + gate_msa * O(attn(RoPE(RMS(Q h)), RoPE(RMS(K h)), V h))
    h = LN(x) * (1 + scale_c) + shift_c                 (affine cross-attn norm)
    x = x + O_c(attn(RMS(Q_c h), RMS(K_c ctx), V_c ctx))
    h = LN(x) * (1 + scale_mlp) + shift_mlp
    x = x + gate_mlp * Down(GELU_tanh(Up h))

with RMS the RMSNorm over all heads of a token (learned weight).

Tensor parallelism (one process per GPU): column-parallel Q/K/V, cross
Q/K/V and FFN-up; attention on the rank's own heads; row-parallel O, cross O
and FFN-down; with sequence parallelism between them (DiTBlock): the INT8
activations are all-gathered before each column-parallel linear and the
row-parallel [L, dim] bf16 partial sums reduce-scattered back to their token
owners, chunk by chunk to overlap the linears; the row-scope RMSNorm of Q and
K adds an all-reduce of the per-token fp32 sums of squares.  A row-parallel layer's input shard must hold whole
256-channel ConvRot groups (its Hadamard rotation and per-token INT8 scale
are taken over the shard), so heads and FFN columns are dealt out in
256-channel units: 40 heads on 8 ranks = 6,6,6,6,4,4,4,4.

Two op backends share the block and its tensor parallelism: KernelOps (the
sm_100a kernels; bf16 activations, INT8 ConvRot linears, INT8 attention) and
TorchOps (fp32 torch with the same dequantized weights and no activation
quantization: the reference's dequantize-then-compute CPU path composed,
validate_compatible.py:110-114, 540-546).
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
import torch.distributed as dist

from .profiling import CUDA_PHASE_PROFILER as PROFILER

GROUP = 256  # ConvRot rotation block


@dataclasses.dataclass(frozen=True)
class BlockConfig:
    dim: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    eps: float = 1e-6

    def __post_init__(self):
        if self.heads * self.head_dim != self.dim:
            raise ValueError("dim must equal heads * head_dim")
        if self.dim % GROUP or self.ffn % GROUP:
            raise ValueError("dim and ffn must be multiples of the 256-channel ConvRot group")
        if self.head_dim != 128:
            raise ValueError("head_dim must be 128 (the attention kernel's tile width)")


def split_units(units: int, parts: int) -> list[int]:
    """units dealt to parts as evenly as possible, the larger shares first."""
    base, extra = divmod(units, parts)
    return [base + (1 if r < extra else 0) for r in range(parts)]


@dataclasses.dataclass(frozen=True)
class ShardPlan:
    world: int
    rank: int
    heads: tuple[int, ...]      # O-projection input heads per rank (whole 256-channel groups)
    ffn: tuple[int, ...]        # FFN columns per rank
    attn: tuple[int, ...] = ()  # attention heads per rank (default: as `heads`)

    def __post_init__(self):
        if not self.attn:
            object.__setattr__(self, "attn", self.heads)

    @property
    def head0(self) -> int:
        return sum(self.heads[: self.rank])

    @property
    def nheads(self) -> int:
        return self.heads[self.rank]

    @property
    def attn0(self) -> int:
        return sum(self.attn[: self.rank])

    @property
    def nattn(self) -> int:
        return self.attn[self.rank]

    @property
    def ffn0(self) -> int:
        return sum(self.ffn[: self.rank])

    @property
    def nffn(self) -> int:
        return self.ffn[self.rank]

    def head_moves(self) -> list[tuple[int, int, int, int]]:
        """(source rank, destination rank, first head, head count) of every
        block of attention outputs that must move to the rank whose O shard
        holds it (both plans are contiguous head ranges in rank order)."""
        moves = []
        a = [sum(self.attn[:r]) for r in range(self.world + 1)]
        o = [sum(self.heads[:r]) for r in range(self.world + 1)]
        for src in range(self.world):
            for dst in range(self.world):
                lo, hi = max(a[src], o[dst]), min(a[src + 1], o[dst + 1])
                if src != dst and hi > lo:
                    moves.append((src, dst, lo, hi - lo))
        return moves


def _interleave(shares: list[int]) -> list[int]:
    """Descending shares reordered big, small, big, small, ... so that each
    larger share sits beside a smaller one."""
    s = sorted(shares, reverse=True)
    out = []
    while s:
        out.append(s.pop(0))
        if s:
            out.append(s.pop())
    return out


def shard_plan(cfg: BlockConfig, world: int, rank: int) -> ShardPlan:
    """O-projection heads in 256-channel units, larger and smaller shares
    alternating; attention heads split evenly when the head count allows
    (then each larger O shard takes the missing heads from its neighbour's
    attention output), else equal to the O shards."""
    heads_per_unit = GROUP // cfg.head_dim
    head_units = cfg.heads // heads_per_unit
    ffn_units = cfg.ffn // GROUP
    if world > head_units:
        raise ValueError(f"{world} ranks exceed the {head_units} 256-channel head groups")
    heads = tuple(u * heads_per_unit for u in _interleave(split_units(head_units, world)))
    attn = tuple([cfg.heads // world] * world) if cfg.heads % world == 0 else heads
    return ShardPlan(world, rank, heads, tuple(u * GROUP for u in split_units(ffn_units, world)),
                     attn)


# ------------------------------------------------------------- weights --

def hadamard256(device=None, dtype=torch.float32) -> torch.Tensor:
    """The orthogonal, symmetric 256-point ConvRot rotation kron(M, M, M, M),
    M = 1/2 [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]
    (kernel/csrc/turing/convrot_quant.cu:104-116)."""
    m = 0.5 * torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
                           dtype=torch.float64)
    h = m
    for _ in range(3):
        h = torch.kron(h, m)
    return h.to(device=device, dtype=dtype)


@dataclasses.dataclass
class QuantLinear:
    """A ConvRot W8A8 linear y = x W^T + b: weight rotated per 256-column
    block (W H, H the rotation above, so that (W H)(H x) = W x) and quantized
    per output channel to INT8 with a fp32 scale."""
    weight: torch.Tensor             # int8 [N, K]
    scale: torch.Tensor              # fp32 [N]
    bias: Optional[torch.Tensor]     # fp32 [N] or None

    @staticmethod
    def from_float(w: torch.Tensor, bias: Optional[torch.Tensor]) -> "QuantLinear":
        n, k = w.shape
        h = hadamard256(w.device)
        wr = (w.float().reshape(n, k // GROUP, GROUP) @ h).reshape(n, k)
        s = wr.abs().amax(dim=1).clamp_min(1e-12) / 127.0
        q = torch.round(wr / s[:, None]).clamp_(-127, 127).to(torch.int8)
        return QuantLinear(q.contiguous(), s.contiguous(),
                           None if bias is None else bias.float().contiguous())

    def dequantized(self) -> torch.Tensor:
        """The fp32 weight this layer applies to unrotated inputs."""
        n, k = self.weight.shape
        w = self.weight.float() * self.scale[:, None]
        return (w.reshape(n, k // GROUP, GROUP) @ hadamard256(w.device)).reshape(n, k)


def _randn(shape, seed: int, device, std: float) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


@dataclasses.dataclass
class BlockWeights:
    qkv: QuantLinear          # rows: q, k, v of the rank's attention heads
    o: QuantLinear            # columns: the rank's O-projection heads; bias on rank 0 only
    cq: QuantLinear
    ckv: QuantLinear          # rows: k, v of the rank's heads (applied to the context)
    co: QuantLinear
    up: QuantLinear           # rows: the rank's FFN columns
    down: QuantLinear         # columns: the rank's FFN columns
    norm_q: torch.Tensor      # RMSNorm weights of the rank's attention heads [nattn * head_dim]
    norm_k: torch.Tensor
    cnorm_q: torch.Tensor
    cnorm_k: torch.Tensor
    modulation: torch.Tensor  # [6, dim]: shift/scale/gate (self-attn), shift/scale/gate (FFN)
    cross_norm: torch.Tensor  # [2, dim]: shift, scale of the affine cross-attention LayerNorm


def make_weights(cfg: BlockConfig, plan: ShardPlan, seed: int = 0, device="cpu",
                 dtype=torch.bfloat16) -> BlockWeights:
    """Random-init weights N(0, 0.02), generated whole
    from per-tensor seeds on every rank and sliced to the rank's shard, then
    ConvRot W8A8-quantized; AdaLN modulation ~N(0, 1)."""
    D, d, f = cfg.head_dim, cfg.dim, cfg.ffn
    hs = slice(plan.attn0 * D, (plan.attn0 + plan.nattn) * D)     # attention heads
    os_ = slice(plan.head0 * D, (plan.head0 + plan.nheads) * D)   # O-projection heads
    fs = slice(plan.ffn0, plan.ffn0 + plan.nffn)
    root = plan.rank == 0

    def w(i, shape):
        return _randn(shape, seed * 1000 + i, device, 0.02)

    def col(ws, bs):  # column-parallel: output rows of the rank
        return QuantLinear.from_float(torch.cat([x[hs] for x in ws]), torch.cat([b[hs] for b in bs]))

    wq, wk, wv, wo = (w(i, (d, d)) for i in range(4))
    bq, bk, bv, bo = (w(10 + i, (d,)) for i in range(4))
    cwq, cwk, cwv, cwo = (w(20 + i, (d, d)) for i in range(4))
    cbq, cbk, cbv, cbo = (w(30 + i, (d,)) for i in range(4))
    up, down = w(40, (f, d)), w(41, (d, f))
    bup, bdown = w(42, (f,)), w(43, (d,))
    norms = [1.0 + w(50 + i, (d,)) for i in range(4)]
    weights = BlockWeights(
        qkv=col([wq, wk, wv], [bq, bk, bv]),
        o=QuantLinear.from_float(wo[:, os_], bo if root else None),
        cq=col([cwq], [cbq]),
        ckv=col([cwk, cwv], [cbk, cbv]),
        co=QuantLinear.from_float(cwo[:, os_], cbo if root else None),
        up=QuantLinear.from_float(up[fs], bup[fs]),
        down=QuantLinear.from_float(down[:, fs], bdown if root else None),
        norm_q=norms[0][hs].to(dtype), norm_k=norms[1][hs].to(dtype),
        cnorm_q=norms[2][hs].to(dtype), cnorm_k=norms[3][hs].to(dtype),
        modulation=_randn((6, d), seed * 1000 + 60, device, 1.0).to(dtype),
        cross_norm=w(61, (2, d)).to(dtype),
    )
    return weights


def rope_freqs(tokens: int, head_dim: int, seed: int = 0, device="cpu",
               dtype=torch.bfloat16) -> torch.Tensor:
    """Per-token 2x2 rotations [1, tokens, 1, head_dim / 2, 2, 2] of random
    angles (the layout the fused Q/K prologue reads; interleaved pairs)."""
    g = torch.Generator(device=device).manual_seed(seed)
    ang = torch.rand((1, tokens, 1, head_dim // 2, 1, 1), generator=g, device=device) * 6.283
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.cat([torch.cat([c, -s], -1), torch.cat([s, c], -1)], -2).to(dtype)


# ------------------------------------------------------------ backends --
#
# A backend turns a [rows, K] activation into the form its linears take
# (`quantize`: a list of row-aligned tensors, which the block may all-gather
# across ranks) and applies a QuantLinear to that form (`linear_q`).

class KernelOps:
    """The sm_100a kernels of this package."""

    def __init__(self):
        from . import _C
        from .turing_sage import core, quant

        self._C, self._core, self._quant = _C, core, quant
        self.launches = 0
        self.event_pair = None  # CUDA events recorded around the self-attention kernel

    def ln_adaln(self, x, scale, shift, eps):
        self.launches += 1
        return self._C.turing_layer_norm_adaln(x[None], scale[None, None], shift[None, None],
                                               eps)[0]

    def quantize(self, x):
        """ConvRot INT8 codes [rows, K] and per-token scales [rows, 1]."""
        self.launches += 1
        return list(self._C.turing_bf16_int8_convrot_quantize(x))

    def gelu_quantize(self, u):
        self.launches += 1
        return list(self._C.turing_bf16_gelu_int8_convrot_quantize(u))

    def linear_q(self, act, layer: QuantLinear, out=None):
        self.launches += 1
        return self._C.turing_int8_linear(act[0], layer.weight, act[1], layer.scale, layer.bias,
                                          out=out)

    def sum_squares(self, t):
        self.launches += 1
        return self._quant.row_sum_squares(t[None], tensor_layout="NHD")[0]

    def qk_prepare(self, q, k, v, qn, kn, freqs, rot_dim, q_rrms, k_rrms, eps):
        """Normalize, rotate and quantize q [Lq, H, D] and k [Lk, H, D] (views)
        once; v [Lk, H, D] may be a strided view (unit channel stride)."""
        self.launches += 1 if q_rrms is not None else 2
        q8, qs, k8, ks = self._quant.rms_rope_per_warp_int8(
            q[None], k[None], qn, kn, freqs, epsilon=eps, rot_dim=rot_dim, tensor_layout="NHD",
            norm_scope="row", split_half=False, rotate_qk=False, stabilize_k=False,
            query_rrms=None if q_rrms is None else q_rrms[None],
            key_rrms=None if k_rrms is None else k_rrms[None])
        return (q8, qs, k8, ks, v[None])

    def attend_rows(self, state, r0: int, r1: int, mark=False, out=None):
        """Attention of query rows [r0, r1) (r0 a multiple of 16) of a
        prepared state -> [r1 - r0, H * D] in V's dtype (into `out`, a
        row block of a larger buffer, when given)."""
        q8, qs, k8, ks, v = state
        self.launches += 1
        if (r0, r1) != (0, q8.size(1)):
            q8 = q8[:, r0:r1]
            tiles = (r1 - r0 + 63) // 64 * 4
            t0 = r0 // 16
            part = qs[:, :, t0:t0 + tiles]
            if part.size(2) < tiles:  # the last 64-token block of the sequence
                part = torch.nn.functional.pad(part, (0, tiles - part.size(2)), value=1.0)
            qs = part
        if mark and self.event_pair is not None:
            self.event_pair[0].record()
        res = self._core.sageattn_prequantized(
            q8.contiguous(), qs.contiguous(), k8, ks, v, tensor_layout="NHD",
            output=None if out is None else out.view(1, r1 - r0, q8.size(2), q8.size(3)))
        if mark and self.event_pair is not None:
            self.event_pair[1].record()
        return res.reshape(r1 - r0, -1)

    def gated_add_(self, x, y, gate):
        """x = bf16(x + y * gate) in place (one kernel, 16-byte vectors)."""
        self.launches += 1
        return self._C.gated_residual_add_(x, y, gate)


class TorchOps:
    """fp32 torch reference with the dequantized weights (activations are not
    quantized)."""
    launches = 0

    def __init__(self):
        self._w: dict[int, torch.Tensor] = {}

    def _dense(self, layer: QuantLinear):
        key = id(layer)
        if key not in self._w:
            self._w[key] = layer.dequantized()
        return self._w[key]

    @staticmethod
    def ln_adaln(x, scale, shift, eps):
        x = x.float()
        return torch.nn.functional.layer_norm(x, (x.size(-1),), eps=eps) * (1 + scale.float()) \
            + shift.float()

    @staticmethod
    def quantize(x):
        return [x.float()]

    @staticmethod
    def gelu_quantize(u):
        return [torch.nn.functional.gelu(u.float(), approximate="tanh")]

    def linear_q(self, act, layer, out=None):
        y = act[0] @ self._dense(layer).t()
        y = y + layer.bias if layer.bias is not None else y
        if out is not None:
            out.copy_(y)
            return out
        return y

    @staticmethod
    def sum_squares(t):
        return t.float().pow(2).sum(dim=(1, 2))

    @staticmethod
    def qk_prepare(q, k, v, qn, kn, freqs, rot_dim, q_rrms, k_rrms, eps):
        def norm_rope(t, w, rrms):
            n = t.float() * rrms[:, None, None] * w.float().view(1, t.size(1), -1)
            if rot_dim:
                f = freqs.float()[0, :, 0]                       # [L, pairs, 2, 2]
                pairs = n.view(n.size(0), n.size(1), -1, 2)       # [L, H, pairs, 2]
                n = torch.einsum("lprc,lhpc->lhpr", f, pairs).reshape(n.shape)
            return n
        if q_rrms is None:
            q_rrms = torch.rsqrt(TorchOps.sum_squares(q) / (q.size(1) * q.size(2)) + eps)
            k_rrms = torch.rsqrt(TorchOps.sum_squares(k) / (k.size(1) * k.size(2)) + eps)
        return (norm_rope(q, qn, q_rrms).transpose(0, 1), norm_rope(k, kn, k_rrms).transpose(0, 1),
                v.float().transpose(0, 1))

    @staticmethod
    def attend_rows(state, r0, r1, mark=False, out=None):
        qf, kf, vf = state
        res = torch.nn.functional.scaled_dot_product_attention(qf[:, r0:r1], kf, vf)
        res = res.transpose(0, 1).reshape(r1 - r0, -1)
        if out is not None:
            out.copy_(res)
            return out
        return res

    @staticmethod
    def gated_add_(x, y, gate):
        return x.addcmul_(y.to(x.dtype), gate.to(x.dtype)) if gate is not None \
            else x.add_(y.to(x.dtype))


# --------------------------------------------------------------- block --

def token_chunks(L: int, world: int, max_chunks: int = 4) -> int:
    """Number of token chunks C of the sequence-parallel layout and of the
    block's pipeline: the largest C <= max_chunks with L divisible by
    C * world and chunk starts on 16-token boundaries (query tiles of the
    attention), preferring C > 1 on several ranks; 1 on one rank."""
    if world == 1:
        return 1
    if L % world:
        raise ValueError(f"{L} tokens do not split evenly over {world} ranks")
    ok = [c for c in range(1, max_chunks + 1) if L % (c * world) == 0 and (L // c) % 16 == 0]
    return max(ok) if ok else 1


def attention_launches(L: int, sms: int = 148, tile: int = 256,
                       split: Optional[int] = None) -> list[tuple[int, int]]:
    """Query-row ranges of the self-attention launches: two, split at a
    multiple of sms * tile rows when that is near L/2 (each launch then fills
    whole waves of the attention kernel's 256-row CTAs on every head count;
    L = 75600 splits at 37888), else one launch."""
    if split is None:
        split = sms * tile
        if abs(2 * split - L) * 8 > L:
            return [(0, L)]
    return [(0, split), (split, L)] if 0 < split < L else [(0, L)]


def local_rows(L: int, world: int, rank: int, chunks: int) -> torch.Tensor:
    """Token indices a rank owns in the sequence-parallel layout: in each of
    the `chunks` equal token chunks, the rank's 1/world slice."""
    piece = L // (chunks * world)
    return torch.cat([torch.arange(c * (L // chunks) + rank * piece,
                                   c * (L // chunks) + (rank + 1) * piece) for c in range(chunks)])


def token_shards(L: int, world: int, block: int = 64) -> list[tuple[int, int]]:
    """Contiguous token ranges of the all-to-all layout, in rank order: whole
    64-token blocks (the K quantizer's tile and four Q warp tiles, so every
    rank's Q/K codes and scales are the one-rank ones) dealt as evenly as
    possible, larger shares first; the last range ends at L.  L = 75600 on 8
    ranks: 6 x 9472, 9408, 9360 tokens."""
    blocks = (L + block - 1) // block
    if blocks < world:
        raise ValueError(f"{L} tokens give fewer 64-token blocks than {world} ranks")
    bounds, t = [], 0
    for share in split_units(blocks, world):
        bounds.append((t, min(t + share * block, L)))
        t = bounds[-1][1]
    return bounds


@dataclasses.dataclass(frozen=True)
class SeqShards:
    """All-to-all sequence parallelism: rank `rank` of `world` owns tokens
    bounds[rank] for every norm, linear and the cross-attention (full
    weights on every rank), and heads [rank * H / world, (rank + 1) * H /
    world) of the self-attention over all tokens; two all-to-alls per block
    move the INT8 Q/K codes, their scales and V to the head owners and the
    attention output back to the token owners."""
    world: int
    rank: int
    bounds: tuple[tuple[int, int], ...]
    group: object = None

    @staticmethod
    def make(L: int, world: int, rank: int, group=None) -> "SeqShards":
        return SeqShards(world, rank, tuple(token_shards(L, world)), group)

    @property
    def sizes(self) -> list[int]:
        return [b - a for a, b in self.bounds]


class DiTBlock:
    """One Wan2.1-style block on one tensor-parallel rank.

    Sequence-parallel layout (Megatron-SP): between the attention / FFN
    sub-blocks every rank holds only its own tokens of x (`local_rows`), runs
    LayerNorm+AdaLN, the ConvRot quantizer and the residual adds on them, and
    all-gathers the INT8 codes and scales (half the bytes of bf16) before each
    column-parallel linear; each row-parallel linear's [tokens, dim] partial
    sums are reduce-scattered back to the token owners.

    The block runs as stages over C token chunks (`token_chunks`), each stage
    issuing its work for every chunk before the next stage waits on any
    chunk's collective, so a chunk's all-gather / reduce-scatter (on NCCL's
    stream) overlaps the following chunks' linears.  Self-attention runs as
    wave-aligned launches over query rows (`attention_launches`) after one
    Q/K prologue over the whole sequence; a chunk whose rows are finished goes
    through O and starts its reduce-scatter under the next launch.  Cross-
    attention and the FFN are independent per token and run per chunk.
    `group` is the process group (None: one rank); `attn_split` overrides the
    query row at which self-attention splits (tests).

    With `seq` (SeqShards; `plan` is then the one-rank plan and `weights`
    the full weights) the block runs all-to-all sequence parallel instead:
    this rank's tokens go through every norm, linear and the cross-attention
    as on one GPU, and the self-attention of its heads over all tokens sits
    between two all-to-alls (`_heads_exchange`; `_tokens_exchange_start`, one
    per attention launch so a launch's rows travel under the next launch, and
    `_tokens_exchange_finish`).  Every
    output row is then the one-rank block's row bit for bit.
    """

    def __init__(self, cfg: BlockConfig, weights: BlockWeights, plan: ShardPlan, ops,
                 group=None, max_chunks: int = 4, attn_split: Optional[int] = None,
                 seq: Optional[SeqShards] = None):
        self.cfg, self.w, self.plan, self.ops, self.group = cfg, weights, plan, ops, group
        self.max_chunks, self.attn_split, self.seq = max_chunks, attn_split, seq
        if seq is not None:
            if plan.world != 1:
                raise ValueError("all-to-all sequence parallelism takes the one-rank plan")
            if cfg.heads % seq.world:
                raise ValueError(f"{cfg.heads} heads do not split evenly over {seq.world} ranks")

    # ----- collectives (identity on one rank)
    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.plan.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def _gather(self, act: list) -> tuple[list, list]:
        """Start all-gathering one chunk's local rows of each tensor in act."""
        if self.plan.world == 1:
            return act, []
        out, works = [], []
        for t in act:
            full = torch.empty((t.size(0) * self.plan.world,) + tuple(t.shape[1:]),
                               dtype=t.dtype, device=t.device)
            works.append(dist.all_gather_into_tensor(full, t.contiguous(), group=self.group,
                                                     async_op=True))
            out.append(full)
        return out, works

    def _scatter(self, y: torch.Tensor):
        """Start reduce-scattering one chunk's [rows, dim] partial sums."""
        if self.plan.world == 1:
            return y, None
        out = torch.empty((y.size(0) // self.plan.world, y.size(1)), dtype=y.dtype,
                          device=y.device)
        return out, (dist.reduce_scatter_tensor(out, y, group=self.group, async_op=True), y)

    @staticmethod
    def _wait(works):
        for wk in works:
            wk.wait()

    def _to_o_heads(self, att: torch.Tensor) -> torch.Tensor:
        """[rows, nattn * D] attention output of this rank's attention heads ->
        [rows, nheads * D] input of its O shard: blocks of heads move between
        ranks point to point (plan.head_moves)."""
        p, D = self.plan, self.cfg.head_dim
        moves = p.head_moves()
        if not moves:
            return att
        rows = att.size(0)
        ops, keep, recv = [], [], []
        for src, dst, h, n in moves:
            if src == p.rank:
                blk = att[:, (h - p.attn0) * D:(h - p.attn0 + n) * D].contiguous()
                keep.append(blk)
                ops.append(dist.P2POp(dist.isend, blk, dst, group=self.group))
            elif dst == p.rank:
                buf = torch.empty((rows, n * D), dtype=att.dtype, device=att.device)
                recv.append((h, buf))
                ops.append(dist.P2POp(dist.irecv, buf, src, group=self.group))
        for req in dist.batch_isend_irecv(ops):
            req.wait()
        out = torch.empty((rows, p.nheads * D), dtype=att.dtype, device=att.device)
        lo, hi = max(p.attn0, p.head0), min(p.attn0 + p.nattn, p.head0 + p.nheads)
        if hi > lo:
            out[:, (lo - p.head0) * D:(hi - p.head0) * D] = att[:, (lo - p.attn0) * D:(hi - p.attn0) * D]
        for h, buf in recv:
            out[:, (h - p.head0) * D:(h - p.head0) * D + buf.size(1)] = buf
        return out

    @staticmethod
    def _all_to_all(recv, send, out_splits, in_splits, group, async_op=False):
        """dist.all_to_all_single with NCCL's contract checked on every
        backend: the split sizes count rows of dim 0 of each tensor."""
        if recv.size(0) != sum(out_splits) or send.size(0) != sum(in_splits):
            raise ValueError("all-to-all split sizes must sum to dim 0 of the tensors")
        return dist.all_to_all_single(recv, send, out_splits, in_splits, group=group,
                                      async_op=async_op)

    def _heads_exchange(self, state):
        """All-to-all of the prepared self-attention operands of this rank's
        tokens (all heads) -> those of this rank's heads (all tokens): the
        INT8 Q/K codes, their per-tile scales and V (KernelOps), or the fp32
        Q/K/V (TorchOps).  Chunks are sent in token-shard order, so what
        arrives is already in token order."""
        seq, D = self.seq, self.cfg.head_dim
        W, sizes, me = seq.world, seq.sizes, seq.rank
        nh, L, Lr = self.cfg.heads // W, sum(seq.sizes), seq.sizes[seq.rank]
        works = []

        def tokens_nhd(t):  # [Lr, H, D] (any strides, unit channel stride) -> [L, nh, D]
            send = t.reshape(Lr, W, nh, D).permute(1, 0, 2, 3).reshape(W * Lr, nh, D)
            recv = torch.empty((L, nh, D), dtype=t.dtype, device=t.device)
            works.append(self._all_to_all(recv, send, sizes, [Lr] * W, seq.group, True))
            return recv

        def tokens_hnd(t):  # [H, Lr, D] -> flat pieces of [nh, L_src, D]
            send = t.reshape(W, nh * Lr * D).contiguous()
            recv = torch.empty((nh * L * D,), dtype=t.dtype, device=t.device)
            works.append(self._all_to_all(recv, send.view(-1), [nh * n * D for n in sizes],
                                          [nh * Lr * D] * W, seq.group, True))
            return recv

        def tiles(sc, per_block):  # [1, H, n_me] per-tile scales -> list of [nh, n_src] pieces
            counts = [(n + 63) // 64 * per_block for n in sizes]
            assert sc.size(-1) == counts[me]
            recv = torch.empty((nh * sum(counts),), dtype=sc.dtype, device=sc.device)
            works.append(self._all_to_all(recv, sc.contiguous().view(-1),
                                          [nh * n for n in counts], [nh * counts[me]] * W,
                                          seq.group, True))
            return recv, counts

        if isinstance(self.ops, KernelOps):
            q8, qs, k8, ks, v = state
            q_full, k_full, v_full = tokens_nhd(q8[0]), tokens_nhd(k8[0]), tokens_nhd(v[0])
            (qr, qc), (kr, kc) = tiles(qs, 4), tiles(ks, 1)
            self._wait(works)

            def join(recv, counts):
                parts = recv.split([nh * n for n in counts])
                return torch.cat([p.view(nh, n) for p, n in zip(parts, counts)], dim=1)[None]

            return (q_full[None], join(qr, qc), k_full[None], join(kr, kc), v_full[None])
        qf, kf, vf = state
        out = [tokens_hnd(t) for t in (qf, kf, vf)]
        self._wait(works)

        def join_hnd(recv):
            parts = recv.split([nh * n * D for n in sizes])
            return torch.cat([p.view(nh, n, D) for p, n in zip(parts, sizes)], dim=1)

        return tuple(join_hnd(r) for r in out)

    def _tokens_exchange_start(self, att: torch.Tensor, a0: int, a1: int):
        """Starts the all-to-all that returns rows [a0, a1) of the
        self-attention output [L, nh * D] of this rank's heads to the ranks
        owning those tokens (async: it runs under the next attention launch).
        Returns (work, received rows, this rank's row range inside its shard)."""
        seq = self.seq
        W, me = seq.world, seq.rank
        send = [max(0, min(a1, t1) - max(a0, t0)) for t0, t1 in seq.bounds]
        t0, t1 = seq.bounds[me]
        r0, r1 = max(a0, t0), min(a1, t1)
        m = max(0, r1 - r0)
        recv = torch.empty((W * m, att.size(1)), dtype=att.dtype, device=att.device)
        work = self._all_to_all(recv, att[a0:a1], [m] * W, send, seq.group, async_op=True)
        return work, recv, (r0 - t0, r0 - t0 + m)

    def _tokens_exchange_finish(self, parts, width: int) -> torch.Tensor:
        """Waits for the exchanges of _tokens_exchange_start and assembles
        this rank's [Lr, H * D] attention output (heads in rank order)."""
        seq = self.seq
        W, Lr = seq.world, seq.sizes[seq.rank]
        out = None
        for work, recv, (r0, r1) in parts:
            work.wait()
            if out is None:
                out = torch.empty((Lr, W, width), dtype=recv.dtype, device=recv.device)
            if r1 > r0:
                out[r0:r1] = recv.view(W, r1 - r0, width).permute(1, 0, 2)
        return out.view(Lr, W * width)

    def _rrms(self, t: torch.Tensor) -> Optional[torch.Tensor]:
        """Row RRMS over the heads of every rank (None: one rank, the fused
        prologue computes it)."""
        if self.plan.world == 1 and isinstance(self.ops, KernelOps):
            return None
        s = self._all_reduce(self.ops.sum_squares(t).float().contiguous())
        return torch.rsqrt(s / self.cfg.dim + self.cfg.eps)

    def forward(self, x_local: torch.Tensor, ctx: torch.Tensor, freqs: torch.Tensor,
                L: Optional[int] = None, branches=("self", "cross", "ffn"),
                trace: Optional[list] = None) -> torch.Tensor:
        """x_local: this rank's tokens of x (`local_rows`, or `seq.bounds`
        with SeqShards; all of x on one rank), ctx [Lc, dim] (every rank),
        freqs [1, L, 1, head_dim/2, 2, 2] (all tokens).  Returns this rank's
        tokens of the block output.  `branches` names the residual branches
        added to x (all by default; tests hold each branch alone to a bound)
        and `trace`, when given, receives (branch, chunk, branch output)
        before each residual add."""
        c, w, ops, N = self.cfg, self.w, self.ops, self.plan.world
        D, nh = c.head_dim, self.plan.nattn
        seq = self.seq
        if seq is None:
            L = x_local.size(0) * N if L is None else L
            Ll, fr = L, freqs      # tokens whose Q/K/V this rank computes
        else:
            L = seq.bounds[-1][1]
            t0, t1 = seq.bounds[seq.rank]
            if x_local.size(0) != t1 - t0:
                raise ValueError("x_local must hold this rank's token shard")
            Ll, fr = t1 - t0, freqs[:, t0:t1]
        C = token_chunks(Ll, N, self.max_chunks)
        rows, piece = Ll // C, Ll // (C * N)
        Lc = ctx.size(0)
        m = w.modulation
        x = x_local.clone()
        xs = [x[i * piece:(i + 1) * piece] for i in range(C)]      # views of x
        full_dtype = torch.bfloat16 if isinstance(ops, KernelOps) else torch.float32

        def residual(name, i, y, gate):
            if trace is not None:
                trace.append((name, i, y.clone()))
            if name in branches:
                ops.gated_add_(xs[i], y, gate)

        # Q/K/V of the whole sequence: per chunk LayerNorm+AdaLN, quantize,
        # all-gather, GEMM into the chunk's rows.
        with PROFILER.phase("dit.norm_qkv"):
            gathered = [self._gather(ops.quantize(ops.ln_adaln(xi, m[1], m[0], c.eps)))
                        for xi in xs]
            qkv = torch.empty((Ll, 3 * nh * D), dtype=full_dtype, device=x.device)
            for i, (act, works) in enumerate(gathered):
                self._wait(works)
                ops.linear_q(act, w.qkv, out=qkv[i * rows:(i + 1) * rows])
            del gathered
        qkv = qkv.view(Ll, 3, nh, D)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        with PROFILER.phase("dit.qk_prologue"):
            state = ops.qk_prepare(q, k, v, w.norm_q, w.norm_k, fr, D, self._rrms(q),
                                   self._rrms(k), c.eps)
        nha = nh                   # heads of this rank's self-attention
        if seq is not None:
            with PROFILER.phase("dit.heads_all_to_all"):
                state = self._heads_exchange(state)
            nha = c.heads // seq.world
        # Self-attention in wave-aligned launches; every chunk whose rows are
        # done goes through O and starts its reduce-scatter while the next
        # attention launch runs (tensor parallel).  All-to-all: the output
        # returns to the token owners after the last launch.
        att = torch.empty((L, nha * D), dtype=full_dtype, device=x.device)
        pending, done = [], 0
        exchanges = []
        with PROFILER.phase("dit.self_attention" if seq is not None else "dit.self_attention_o"):
            for a0, a1 in attention_launches(L, split=self.attn_split):
                ops.attend_rows(state, a0, a1, mark=a1 == L, out=att[a0:a1])
                if seq is not None:  # these rows go home under the next launch
                    exchanges.append(self._tokens_exchange_start(att, a0, a1))
                while seq is None and done < C and (done + 1) * rows <= a1:
                    blk = att[done * rows:(done + 1) * rows]
                    pending.append(self._scatter(
                        ops.linear_q(ops.quantize(self._to_o_heads(blk)), w.o)))
                    done += 1
        if seq is not None:
            with PROFILER.phase("dit.tokens_all_to_all"):
                att = self._tokens_exchange_finish(exchanges, nha * D)
            with PROFILER.phase("dit.o_proj"):
                pending.append(self._scatter(ops.linear_q(ops.quantize(att), w.o)))
        del state, qkv, q, k, v, att

        # Cross-attention: the context's K/V once, then per chunk.
        with PROFILER.phase("dit.cross_attention"):
            kv = ops.linear_q(ops.quantize(ctx), w.ckv).view(Lc, 2, nh, D)
            k_rrms = self._rrms(kv[:, 0])
            gathered = []
            for i, (y, job) in enumerate(pending):
                if job is not None:
                    job[0].wait()
                residual("self", i, y, m[2])
                gathered.append(self._gather(ops.quantize(ops.ln_adaln(xs[i], w.cross_norm[1],
                                                                       w.cross_norm[0], c.eps))))
            # Q of every chunk first, so the cross-rank RMS of all chunks is one
            # all-reduce (a collective queues behind the chunks' gathers).
            qcs = []
            for i, (act, works) in enumerate(gathered):
                self._wait(works)
                qcs.append(ops.linear_q(act, w.cq).view(rows, nh, D))
            q_rrms = [None] * C
            if N > 1 or not isinstance(ops, KernelOps):
                sums = self._all_reduce(torch.cat([ops.sum_squares(qc).float() for qc in qcs]))
                q_rrms = list(torch.rsqrt(sums / c.dim + c.eps).split(rows))
            pending = []
            for i, qc in enumerate(qcs):
                st = ops.qk_prepare(qc, kv[:, 0], kv[:, 1], w.cnorm_q, w.cnorm_k, None, 0,
                                    q_rrms[i], k_rrms, c.eps)
                att = ops.attend_rows(st, 0, rows)
                pending.append(self._scatter(
                    ops.linear_q(ops.quantize(self._to_o_heads(att)), w.co)))
            del qcs

        # Feed-forward per chunk.
        with PROFILER.phase("dit.ffn"):
            gathered = []
            for i, (y, job) in enumerate(pending):
                if job is not None:
                    job[0].wait()
                residual("cross", i, y, None)
                gathered.append(self._gather(ops.quantize(ops.ln_adaln(xs[i], m[4], m[3], c.eps))))
            pending = []
            for i, (act, works) in enumerate(gathered):
                self._wait(works)
                u = ops.linear_q(act, w.up)
                pending.append(self._scatter(ops.linear_q(ops.gelu_quantize(u), w.down)))
            for i, (y, job) in enumerate(pending):
                if job is not None:
                    job[0].wait()
                residual("ffn", i, y, m[5])
        PROFILER.complete_attention((L, c.dim))
        return x

    def ops_count(self, L: int, Lc: int) -> float:
        """Algorithmic operations of the whole block (all ranks): 2 per
        multiply-add of every linear and of QK^T and PV."""
        d, f, H, D = self.cfg.dim, self.cfg.ffn, self.cfg.heads, self.cfg.head_dim
        lin = 2 * L * d * (3 * d) + 2 * L * d * d + 2 * 2 * L * d * d + 2 * Lc * d * 2 * d \
            + 2 * 2 * L * d * f
        attn = 4 * H * L * L * D + 4 * H * L * Lc * D
        return float(lin + attn)


@torch.no_grad()
def reference_rows(cfg: BlockConfig, w: BlockWeights, x: torch.Tensor, ctx: torch.Tensor,
                   freqs: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """The fp32 reference block (TorchOps' arithmetic: dequantized weights,
    unquantized activations) at token rows `idx` only, from one-rank weights
    `w` and all tokens of x: K and V are computed for every token, Q and the
    rest of the block for the sampled rows.  Equals
    DiTBlock(cfg, w, plan, TorchOps()).forward(x, ctx, freqs)[idx] up to fp32
    summation order; used to check multi-GPU outputs on a row sample."""
    ops, m, eps = TorchOps(), w.modulation, cfg.eps
    d, H, D = cfg.dim, cfg.heads, cfg.head_dim
    x = x.float()
    L, R = x.size(0), idx.numel()

    def lin(a, layer, rows=None):
        wt = ops._dense(layer) if rows is None else ops._dense(layer)[rows]
        y = a @ wt.t()
        if layer.bias is not None:
            y = y + (layer.bias if rows is None else layer.bias[rows])
        return y

    def norm_rope(t, weight, f):  # t [n, H, D]; row RMSNorm over all heads, RoPE by f
        rrms = torch.rsqrt(t.pow(2).sum(dim=(1, 2)) / d + eps)
        n = t * rrms[:, None, None] * weight.float().view(1, H, D)
        if f is not None:
            pairs = n.view(n.size(0), H, D // 2, 2)
            n = torch.einsum("lprc,lhpc->lhpr", f.float()[0, :, 0], pairs).reshape(n.shape)
        return n

    h = ops.ln_adaln(x, m[1], m[0], eps)
    q = lin(h[idx], w.qkv, slice(0, d)).view(R, H, D)
    k = lin(h, w.qkv, slice(d, 2 * d)).view(L, H, D)
    v = lin(h, w.qkv, slice(2 * d, 3 * d)).view(L, H, D)
    del h
    q, k = norm_rope(q, w.norm_q, freqs[:, idx]), norm_rope(k, w.norm_k, freqs)
    a = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1),
                                                         v.transpose(0, 1))
    del k, v
    xr = x[idx] + lin(a.transpose(0, 1).reshape(R, d), w.o) * m[2].float()
    hc = ops.ln_adaln(xr, w.cross_norm[1], w.cross_norm[0], eps)
    qc = norm_rope(lin(hc, w.cq).view(R, H, D), w.cnorm_q, None)
    kv = lin(ctx.float(), w.ckv).view(ctx.size(0), 2, H, D)
    kc = norm_rope(kv[:, 0], w.cnorm_k, None)
    a = torch.nn.functional.scaled_dot_product_attention(qc.transpose(0, 1), kc.transpose(0, 1),
                                                         kv[:, 1].transpose(0, 1))
    xr = xr + lin(a.transpose(0, 1).reshape(R, d), w.co)
    hf = ops.ln_adaln(xr, m[4], m[3], eps)
    u = torch.nn.functional.gelu(lin(hf, w.up), approximate="tanh")
    return xr + lin(u, w.down) * m[5].float()


def block_ops(cfg: BlockConfig, L: int, Lc: int) -> float:
    return DiTBlock(cfg, None, shard_plan(cfg, 1, 0), None).ops_count(L, Lc)
