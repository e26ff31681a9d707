"""The MMDiT joint block and the denoising step over the W8A8 linear family.

The BASELINE model is the original Qwen-Image MMDiT: 60 joint blocks of
hidden 3072, 24 heads x 128, a GELU-tanh MLP of 12288 and a per-block,
per-stream AdaLN modulation 3072 -> 18432.  No code for it exists in the
reference (its Qwen-Image 2.1 DiT is single-stream, hidden 4096), so it is
assembled here from the reference's operators and model steps:

* per stream (image, text): AdaLN (``modulated_norm``,
  inference/src/models/qwen_image21/numeric.rs:63-108) fused into the QKV
  projection's quantiser, with the per-head Q/K RMSNorm + RoPE
  (``rms_rope``, dit.rs:486-505) fused into its GEMM epilogue;
* joint attention over the text tokens followed by the image tokens (the
  sequence order of ``assemble_sequence``, geometry.rs:143-230), bf16
  scaled-dot-product attention;
* the out-projection and MLP-down with the gated residual
  (``gated_residual``, numeric.rs:110-126) in their GEMM epilogues;
* AdaLN fused into MLP-up's quantiser, GELU-tanh in its epilogue;
* the block loop of ``DiT::forward_original`` (dit.rs:567-757): text
  projection, timestep embedding (numeric.rs:22-50), 3-axis RoPE
  (geometry.rs:65-110), final AdaLN + projection.

The modulation linears of all blocks read the same SiLU(temb) row, so their
weights are stored as one [blocks * 6 * hidden, hidden] matrix per stream and
run as ONE M <= 2 GEMV per stream per step.

Every numeric step goes through an ``ops`` object.  ``NativeOps`` is libw8a8
(imagine_b200.linear) plus torch's scaled-dot-product attention; the tests
run the same model code over a CPU oracle for parity.

Multi-GPU (one process per GPU):

* CFG: the two branches of a CFG step are independent until the combine.
  With 2 or more ranks, ranks [0, W/2) run the conditional branch and
  [W/2, W) the unconditional one; one all-gather between the rank pairs
  (r, r + W/2) gives every rank both predictions (``cfg_model``).
* Sequence parallelism inside a branch (W/2 > 1 ranks, the default): each
  rank of the branch holds the whole weights and a contiguous share of the
  image tokens; per block it writes the k / v of its tokens into its slot of
  a joint k / v buffer, one in-place all-gather fills the others, its
  queries (all text tokens, its image tokens) attend to the whole sequence,
  and every linear is row-local.  The text stream (256 tokens) runs on every
  rank; the modulation GEMV is split by output rows and all-gathered once
  per step; the final image rows are all-gathered.
* Tensor parallelism inside a branch (the alternative): heads are split across
  the ranks of a branch.  QKV and MLP-up are column-parallel (no exchange);
  the out-projection and MLP-down are row-parallel: an all-reduce MAX of the
  row absmax (so every rank quantises its K-slice with the full row's scale),
  an int32 GEMM on the slice, an all-reduce SUM of the exact int32 partials,
  then the dequant + bias + gated-residual epilogue.  The modulation GEMV is
  split by output rows and all-gathered once per step.  Results equal the
  single-GPU model's bit for bit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, fields
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class MMDiTConfig:
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    mlp_hidden: int = 12288
    blocks: int = 60
    latent_channels: int = 16
    patch: int = 2
    context_dim: int = 3072
    time_dim: int = 256
    eps: float = 1e-6
    axes: Tuple[int, int, int] = (16, 56, 56)
    theta: float = 10000.0

    @property
    def in_channels(self) -> int:
        return self.latent_channels * self.patch * self.patch

    @property
    def mod_dim(self) -> int:
        return 6 * self.hidden


# --------------------------------------------------------------------------
# positions, timestep embedding, patches
# --------------------------------------------------------------------------
def sequence_ids(text_tokens: int, h: int, w: int, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Position ids [S, 3] of the text tokens and of the h x w image patches,
    as ``assemble_sequence`` builds them for one image and no references
    (inference/src/models/qwen_image21/geometry.rs:143-230): text token i at
    (i, i, i); the image after it at frame index ``text_tokens`` and centred
    row / column indices."""
    txt = torch.arange(text_tokens, dtype=torch.float32, device=device).unsqueeze(1).expand(text_tokens, 3)
    hh = torch.arange(h, dtype=torch.float32, device=device) - (h - h // 2)
    ww = torch.arange(w, dtype=torch.float32, device=device) - (w - w // 2)
    img = torch.stack([torch.full((h, w), float(text_tokens), device=device),
                       hh.unsqueeze(1).expand(h, w), ww.unsqueeze(0).expand(h, w)], -1)
    return txt.contiguous(), img.reshape(h * w, 3).contiguous()


def rope_freqs(ids: torch.Tensor, axes=(16, 56, 56), theta: float = 10000.0) -> torch.Tensor:
    """Rotations [S, sum(axes) / 2, 2, 2] (fp32) for position ids [S, 3]
    (``PositionEncoding::forward``, geometry.rs:65-110): per axis of width d,
    omega_j = 1 / theta^(j * 2 / d) in float64, angle = pos * omega, and the
    2 x 2 block [[cos, -sin], [sin, cos]]; the axes concatenated along the
    pairs."""
    parts = []
    for axis, dim in enumerate(axes):
        if dim % 2:
            raise ValueError("every RoPE axis needs an even width")
        scale = torch.linspace(0.0, (dim - 2) / dim, dim // 2, dtype=torch.float64, device=ids.device)
        omega = torch.pow(theta, scale).reciprocal()
        ang = torch.einsum("n,d->nd", ids[:, axis].to(torch.float32).double(), omega)
        c, s = torch.cos(ang), torch.sin(ang)
        parts.append(torch.stack([c, -s, s, c], -1).reshape(ids.shape[0], dim // 2, 2, 2).float())
    return torch.cat(parts, dim=1).contiguous()


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0,
                       time_factor: float = 1000.0) -> torch.Tensor:
    """inference/src/models/qwen_image21/numeric.rs:22-50 (fp32)."""
    t = t.to(torch.float32) * time_factor
    half = dim // 2
    freq = torch.exp(torch.arange(half, dtype=torch.float32, device=t.device)
                     * -math.log(max_period) / half)
    args = t.unsqueeze(1) * freq.unsqueeze(0)
    out = torch.cat([torch.cos(args), torch.sin(args)], -1)
    if dim % 2:
        out = torch.cat([out, torch.zeros_like(out[:, :1])], -1)
    return out


def round_timesteps(t: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """numeric.rs:15-20: t * 1000 in the model dtype, / 1000."""
    return (t * 1000).to(dtype).div(1000).to(dtype)


def patchify(x: torch.Tensor, p: int) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/p)(W/p), C p p] (channel, then patch row, then
    patch column)."""
    b, c, h, w = x.shape
    x = x.reshape(b, c, h // p, p, w // p, p).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(b, (h // p) * (w // p), c * p * p)


def unpatchify(x: torch.Tensor, p: int, c: int, h: int, w: int) -> torch.Tensor:
    b = x.shape[0]
    x = x.reshape(b, h // p, w // p, c, p, p).permute(0, 3, 1, 4, 2, 5)
    return x.reshape(b, c, h, w)


# --------------------------------------------------------------------------
# parameters
# --------------------------------------------------------------------------
@dataclass
class Int8Params:
    """One quantised linear: int8 w [N, K], fp32 per-output-channel ws [N],
    bf16 bias [N] (or None)."""
    w: torch.Tensor
    ws: torch.Tensor
    b: Optional[torch.Tensor]

    def to(self, device) -> "Int8Params":
        return Int8Params(self.w.to(device), self.ws.to(device),
                          None if self.b is None else self.b.to(device))


@dataclass
class StreamParams:
    """One stream of a joint block on one rank: QKV rows are this rank's heads
    (q rows, then k rows, then v rows), ``qk_norm`` the per-column RMSNorm
    weight of the q and k columns, ``out`` / ``down`` this rank's K-slice
    (all output channels), ``up`` this rank's output rows."""
    qkv: Int8Params
    qk_norm: torch.Tensor
    out: Int8Params
    up: Int8Params
    down: Int8Params


@dataclass
class BlockParams:
    img: StreamParams
    txt: StreamParams


@dataclass
class MMDiTParams:
    cfg: MMDiTConfig
    tp_rank: int
    tp_world: int
    blocks: List[BlockParams]
    mod_img: Int8Params   # this rank's rows of [blocks * 6 * hidden, hidden]
    mod_txt: Int8Params
    time1: Int8Params     # [hidden, time_dim]
    time2: Int8Params     # [hidden, hidden]
    img_in: Int8Params    # [hidden, in_channels]
    txt_norm: torch.Tensor  # bf16 [context_dim]
    txt_in: Int8Params    # [hidden, context_dim]
    norm_out: Int8Params  # [2 * hidden, hidden]: scale rows, then shift rows
    proj_out: Int8Params  # [in_channels, hidden]

    def to(self, device) -> "MMDiTParams":
        def mv(v):
            if isinstance(v, (Int8Params, StreamParams, BlockParams)):
                return type(v)(**{f.name: mv(getattr(v, f.name)) for f in fields(v)})
            if isinstance(v, torch.Tensor):
                return v.to(device)
            if isinstance(v, list):
                return [mv(e) for e in v]
            return v
        return MMDiTParams(**{f.name: mv(getattr(self, f.name)) for f in fields(self)})

    @property
    def weight_bytes(self) -> int:
        total = 0

        def acc(v):
            nonlocal total
            if isinstance(v, torch.Tensor):
                total += v.numel() * v.element_size()
            elif isinstance(v, (Int8Params, StreamParams, BlockParams)):
                for f in fields(v):
                    acc(getattr(v, f.name))
            elif isinstance(v, list):
                for e in v:
                    acc(e)
        for f in fields(self):
            acc(getattr(self, f.name))
        return total


def _shard(total: int, rank: int, world: int) -> slice:
    if total % world:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    n = total // world
    return slice(rank * n, (rank + 1) * n)


class _Init:
    """Seeded random-init weights ~ N(0, 0.02) (bf16), quantised per output
    channel by ``ops.quantize_weight``; every rank draws the full matrix from
    the same seed and keeps its slice, so shards equal the single-GPU
    weights' slices exactly."""

    def __init__(self, ops, device, seed: int):
        self.ops = ops
        self.device = torch.device(device)
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(seed)

    def randn(self, *shape, std=0.02):
        return (torch.randn(*shape, generator=self.gen, device=self.device) * std).to(torch.bfloat16)

    def linear(self, n, k, rows: Optional[slice] = None, cols: Optional[slice] = None,
               bias=True) -> Int8Params:
        w = self.randn(n, k)
        b = self.randn(n) if bias else None
        q, ws = self.ops.quantize_weight(w)
        del w
        ws = ws.reshape(-1)
        if rows is not None:
            q, ws = q[rows], ws[rows]
            b = b[rows] if b is not None else None
        if cols is not None:
            q = q[:, cols]
        return Int8Params(q.contiguous(), ws.contiguous(), None if b is None else b.contiguous())


def random_params(cfg: MMDiTConfig, ops, device, seed: int = 0, tp_rank: int = 0,
                  tp_world: int = 1) -> MMDiTParams:
    """Random-init weights of the architecture ``cfg`` (this rank's shards)."""
    if cfg.heads % tp_world:
        raise ValueError(f"{cfg.heads} heads do not split over {tp_world} ranks")
    init = _Init(ops, device, seed)
    hd = cfg.heads * cfg.head_dim
    if hd != cfg.hidden:
        raise ValueError("hidden must equal heads * head_dim")
    heads = _shard(hd, tp_rank, tp_world)
    qkv_rows = [slice(i * hd + heads.start, i * hd + heads.stop) for i in range(3)]
    mlp_rows = _shard(cfg.mlp_hidden, tp_rank, tp_world)

    def stream():
        w = init.randn(3 * hd, cfg.hidden)
        b = init.randn(3 * hd)
        q, ws = ops.quantize_weight(w)
        del w
        ws = ws.reshape(-1)
        qkv = Int8Params(torch.cat([q[r] for r in qkv_rows]).contiguous(),
                         torch.cat([ws[r] for r in qkv_rows]).contiguous(),
                         torch.cat([b[r] for r in qkv_rows]).contiguous())
        qn = 1.0 + init.randn(cfg.head_dim, std=0.05).float()
        kn = 1.0 + init.randn(cfg.head_dim, std=0.05).float()
        local_heads = cfg.heads // tp_world
        norm = torch.cat([qn.repeat(local_heads), kn.repeat(local_heads)]).to(torch.bfloat16)
        out = init.linear(cfg.hidden, hd, cols=heads)
        up = init.linear(cfg.mlp_hidden, cfg.hidden, rows=mlp_rows)
        down = init.linear(cfg.hidden, cfg.mlp_hidden, cols=mlp_rows)
        return StreamParams(qkv, norm.contiguous(), out, up, down)

    blocks = []
    for _ in range(cfg.blocks):
        img = stream()
        txt = stream()
        blocks.append(BlockParams(img, txt))
    mod_rows = _shard(cfg.blocks * cfg.mod_dim, tp_rank, tp_world)
    mod_img = init.linear(cfg.blocks * cfg.mod_dim, cfg.hidden, rows=mod_rows)
    mod_txt = init.linear(cfg.blocks * cfg.mod_dim, cfg.hidden, rows=mod_rows)
    return MMDiTParams(
        cfg=cfg, tp_rank=tp_rank, tp_world=tp_world, blocks=blocks, mod_img=mod_img,
        mod_txt=mod_txt, time1=init.linear(cfg.hidden, cfg.time_dim),
        time2=init.linear(cfg.hidden, cfg.hidden), img_in=init.linear(cfg.hidden, cfg.in_channels),
        txt_norm=(1.0 + init.randn(cfg.context_dim, std=0.05).float()).to(torch.bfloat16),
        txt_in=init.linear(cfg.hidden, cfg.context_dim),
        norm_out=init.linear(2 * cfg.hidden, cfg.hidden),
        proj_out=init.linear(cfg.in_channels, cfg.hidden))


# --------------------------------------------------------------------------
# native operators
# --------------------------------------------------------------------------
class NativeOps:
    """The model's numeric steps on libw8a8 (imagine_b200.linear); attention
    is torch's scaled-dot-product attention in bf16 (the library has no
    attention kernel; the reference's own model calls its attention
    routes the same way, dit.rs:506-515)."""

    def __init__(self, attention_backends=None):
        from torch.nn.attention import SDPBackend

        from . import linear

        self.L = linear
        # cuDNN's fused attention first: on B200 it runs the joint attention
        # of the 1600x896 step (B 2, 24 heads, 5856 tokens) in 0.58 ms
        # (1.46 PFLOP/s) against 2.13 ms for torch's flash kernel
        self.attention_backends = attention_backends or [
            SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
            SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]

    def quantize_weight(self, w):
        return self.L.quantize_weight(w)

    def linear(self, x, p: Int8Params, act=None, residual=None, gate=None, input_norm=None,
               eps=1e-6):
        if input_norm is not None:
            return self.L.int8_linear(x, p.w, p.ws, p.b, torch.bfloat16, input_act="rms_norm",
                                      input_act_weight=input_norm, input_act_eps=eps,
                                      output_act=act)
        return self.L.int8_linear(x, p.w, p.ws, p.b, torch.bfloat16, residual=residual,
                                  residual_scale=gate, output_act=act)

    def adaln_linear(self, x, scale, shift, p: Int8Params, act=None, eps=1e-6):
        return self.L.adaln_int8_linear(x, scale, shift, p.w, p.ws, p.b, torch.bfloat16, eps=eps,
                                        output_act=act)

    def adaln_qkv_rope(self, x, scale, shift, p: Int8Params, norm_w, freqs, rope_cols, eps=1e-6):
        return self.L.int8_linear_rms_rope(x, p.w, p.ws, p.b, norm_w, freqs, eps, rope_cols,
                                           modulation=(scale, shift, eps, False))

    def row_absmax(self, x):
        return self.L.row_absmax(x).reshape(-1).contiguous()

    def quantize_given_absmax(self, x, amax):
        q, s = self.L.quantize_int8_rowwise_given_absmax(x, amax)
        return q, s.reshape(-1)

    def gemm_s32(self, q, w):
        return self.L.int8_gemm_s32(q, w)

    def dequant(self, acc, xs, p: Int8Params, residual=None, gate=None, lead=None):
        # the eager dequant order: the one int8_linear (the 1-GPU path) uses
        return self.L.dequantize_int8_linear(acc, xs, p.ws, p.b, torch.bfloat16, dequant="eager",
                                             residual=residual, residual_scale=gate, lead=lead)

    def attention(self, joint, heads: int, head_dim: int):
        """Attention over a joint sequence: joint [B, S, 3 * heads * head_dim]
        (q, k, v columns, read in place) -> [B, S, heads * head_dim]."""
        c = heads * head_dim
        return self.attention_split(joint[..., :c], joint[..., c:], heads, head_dim)

    def attention_split(self, q, kv, heads: int, head_dim: int):
        """q [B, Sq, C] against kv [B, Skv, 2C] (k columns, then v), both read
        in place -> [B, Sq, C]."""
        b, sq, _ = q.shape
        c = heads * head_dim
        qh = q.unflatten(-1, (heads, head_dim)).transpose(1, 2)
        k, v = (kv[..., i * c:(i + 1) * c].unflatten(-1, (heads, head_dim)).transpose(1, 2)
                for i in range(2))
        if self.attention_backends:
            from torch.nn.attention import sdpa_kernel

            with sdpa_kernel(self.attention_backends, set_priority=True):
                o = torch.nn.functional.scaled_dot_product_attention(qh, k, v)
        else:
            o = torch.nn.functional.scaled_dot_product_attention(qh, k, v)
        return o.transpose(1, 2).reshape(b, sq, c)

    def adaln_qkv_rope_split(self, x, scale, shift, p: Int8Params, norm_w, freqs, q_outs, kv_outs,
                             eps=1e-6):
        """``adaln_qkv_rope`` with sample i's q columns written into
        ``q_outs[i]`` [S, C] and its k, v columns into ``kv_outs[i]`` [S, 2C]:
        one modulated quantiser over all rows, then per sample the q rows of
        the weight (RMSNorm + RoPE on every column) and its k, v rows (RMSNorm
        + RoPE on the k columns)."""
        b, s, k = x.shape
        c = p.w.shape[0] // 3
        q, xs = self.L.quantize_int8_rowwise_modulated(x, "adaln", scale, shift, None, eps)
        q = q.reshape(-1, k)
        xs = xs.reshape(-1)
        stream = self.L._stream(x.device)
        halves = ((slice(0, c), q_outs), (slice(c, 3 * c), kv_outs))
        for i in range(b):
            rows = slice(i * s, (i + 1) * s)
            for cols, outs in halves:
                self.L._rms_rope_gemm(q[rows], xs[rows], None, p.w[cols], p.ws[cols],
                                      None if p.b is None else p.b[cols],
                                      norm_w[cols.start:cols.start + c], freqs, eps, c, "eager",
                                      None, None, stream, out=outs[i])

    def joint_attention(self, qkv_t, qkv_i, heads: int, head_dim: int):
        """Joint attention of [text; image] tokens.  qkv_*: [B, S, 3 * heads *
        head_dim] (q, k, v columns).  Returns the text and image outputs
        [B, S, heads * head_dim]."""
        st = qkv_t.shape[1]
        o = self.attention(torch.cat([qkv_t, qkv_i], dim=1), heads, head_dim)
        return o[:, :st], o[:, st:]

    def adaln_qkv_rope_into(self, x, scale, shift, p: Int8Params, norm_w, freqs, rope_cols, outs,
                            eps=1e-6):
        """``adaln_qkv_rope`` with sample i's rows written into ``outs[i]``
        (an [S, N] view, e.g. the sample's rows of a joint q / k / v buffer):
        one modulated quantiser over all rows, then one GEMM per sample."""
        b, s, k = x.shape
        q, xs = self.L.quantize_int8_rowwise_modulated(x, "adaln", scale, shift, None, eps)
        q = q.reshape(-1, k)
        xs = xs.reshape(-1)
        stream = self.L._stream(x.device)
        for i, o in enumerate(outs):
            self.L._rms_rope_gemm(q[i * s:(i + 1) * s], xs[i * s:(i + 1) * s], None, p.w, p.ws,
                                  p.b, norm_w, freqs, eps, rope_cols, "eager", None, None, stream,
                                  out=o)

    def silu(self, x):
        return torch.nn.functional.silu(x)

    def row_parallel_fused(self, q, xs, p: Int8Params, group, residual=None, gate=None, lead=None):
        """The row-parallel linear's int32 GEMM with the reduce-scatter in its
        epilogue (w8a8_gemm_s32_reduce_scatter: each finished partial chunk
        goes to the rank that owns its rows over NVLink), then the finish
        (w8a8_reduce_scatter_finish: the owner sums its rows, applies the
        dequant + bias + gated-residual epilogue and hands its rows to the
        others).  Equals all-reduce(int32) followed by ``dequant`` bit for
        bit."""
        import ctypes

        from . import _native as N
        from .tensor_parallel import _PeerBuffers

        L = self.L
        dev = q.device
        key = (id(group), dev.index)
        peers = getattr(self, "_peers", None)
        if peers is None:
            peers = self._peers = {}
        pb = peers.get(key)
        if pb is None:
            pb = peers[key] = _PeerBuffers(group, dev)
        m, k = q.shape
        n = p.w.shape[0]
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        recvs = pb._mapped("_rs_recv", int(N.LIB.w8a8_reduce_scatter_recv_bytes(m, n, world)), dev)
        stages = pb._mapped("_rs_stage", m * n * 2, dev)
        lead = tuple(lead) if lead is not None else (m,)
        r = rs = None
        rs_rows = 0
        if residual is not None:
            r = residual.reshape(m, n).contiguous()
            rs, rs_rows = L._residual_scale(gate, lead, n, torch.bfloat16, dev)
        b = p.b.contiguous() if p.b is not None else None
        ep = L._epilogue(p.ws, b, r, rs, "eager", None, n, n, rs_rows)
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        epoch = pb.next_epoch()
        stream = L._stream(dev)
        N.check(N.LIB.w8a8_peer_barrier(pb.flag_ptrs, rank, world, epoch, stream))
        N.check(N.LIB.w8a8_gemm_s32_reduce_scatter(L._vp(q), k, L._vp(p.w), k, m, n, k, recvs,
                                                   pb.flag_ptrs, rank, world, epoch, None, stream))
        N.check(N.LIB.w8a8_reduce_scatter_finish(L._vp(xs), ctypes.byref(ep), L._vp(y), N.BF16, n,
                                                 m, n, recvs, stages, pb.flag_ptrs, rank, world,
                                                 epoch, stream))
        return y.reshape(*lead, n)


# --------------------------------------------------------------------------
# the model
# --------------------------------------------------------------------------
class MMDiT:
    """The MMDiT forward on one rank: alone, in a tensor-parallel group
    (``tp_group``, with the weight shards of ``random_params(tp_rank,
    tp_world)``) or in a sequence-parallel group (``sp_group``, whole
    weights)."""

    def __init__(self, params: MMDiTParams, ops, tp_group=None, fused_tp: bool = False,
                 sp_group=None):
        self.p = params
        self.cfg = params.cfg
        self.ops = ops
        self.tp_group = tp_group
        self.tp = params.tp_world
        # sequence parallelism: this rank's share of the image tokens, whole
        # weights (one sample per call)
        self.sp_group = sp_group
        self.sp = dist.get_world_size(sp_group) if sp_group is not None else 1
        self.sp_rank = dist.get_rank(sp_group) if sp_group is not None else 0
        if self.sp > 1 and self.tp > 1:
            raise ValueError("sequence and tensor parallelism are alternatives here")
        # row-parallel reduction fused into the GEMM (peer memory) instead of
        # an NCCL all-reduce of the int32 partials
        self.fused_tp = fused_tp and self.tp > 1 and hasattr(ops, "row_parallel_fused")
        if self.tp > 1 and (tp_group is None or dist.get_world_size(tp_group) != self.tp):
            raise ValueError("the parameters are sharded; pass their tensor-parallel group")
        self._freqs = {}

    # -- helpers -------------------------------------------------------------
    def freqs(self, text_tokens: int, h: int, w: int, device):
        key = (text_tokens, h, w, str(device))
        if key not in self._freqs:
            ids_t, ids_i = sequence_ids(text_tokens, h, w, device)
            self._freqs[key] = (rope_freqs(ids_t, self.cfg.axes, self.cfg.theta),
                                rope_freqs(ids_i, self.cfg.axes, self.cfg.theta))
        return self._freqs[key]

    def _row_parallel(self, x, p: Int8Params, residual, gate):
        """x [B, S, K/tp] (this rank's K-slice; a sample's rows contiguous,
        samples possibly apart) -> [B, S, N] with the gated residual, equal to
        the single-GPU linear bit for bit."""
        lead = x.shape[:-1]
        if self.tp == 1:
            return self.ops.linear(x, p, residual=residual, gate=gate)
        x2 = x.reshape(-1, x.shape[-1])
        amax = self.ops.row_absmax(x2)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.tp_group)
        q, xs = self.ops.quantize_given_absmax(x2, amax)
        if self.fused_tp:
            return self.ops.row_parallel_fused(q, xs, p, self.tp_group, residual=residual,
                                               gate=gate, lead=lead)
        acc = self.ops.gemm_s32(q, p.w)
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.tp_group)
        return self.ops.dequant(acc, xs, p, residual=residual, gate=gate, lead=lead)

    def _gather_cols(self, y):
        """All-gather a [B, N/tp] row-shard of the modulation output."""
        if self.tp == 1:
            return y
        parts = [torch.empty_like(y) for _ in range(self.tp)]
        dist.all_gather(parts, y.contiguous(), group=self.tp_group)
        return torch.cat(parts, dim=-1)

    def _mod_linear(self, s, p: Int8Params):
        """The modulation GEMV of every block: on sequence-parallel ranks each
        computes its share of the output rows and one all-gather joins them."""
        if self.sp == 1:
            return self._gather_cols(self.ops.linear(s, p))
        n = p.w.shape[0]
        rows = _shard(n, self.sp_rank, self.sp)
        mine = self.ops.linear(s, Int8Params(p.w[rows], p.ws[rows],
                                             None if p.b is None else p.b[rows]))
        b = mine.shape[0]
        out = torch.empty((self.sp * b, mine.shape[1]), dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(out, mine.contiguous(), group=self.sp_group)
        return out.reshape(self.sp, b, -1).permute(1, 0, 2).reshape(b, n)

    # -- one joint block -------------------------------------------------------
    @staticmethod
    def _mod_chunks(mod, b, hidden):
        """shift1, scale1, gate1, shift2, scale2, gate2 as [B, 1, hidden]
        tensors, from one block's modulation: [6, B, hidden] (contiguous
        chunks, as ``forward`` lays them out) or [B, 6 * hidden]."""
        if mod.dim() == 2:
            mod = mod.reshape(b, 6, hidden).transpose(0, 1).contiguous()
        return tuple(mod[j].unsqueeze(1) for j in range(6))

    def block(self, bp: BlockParams, img, txt, mod_i, mod_t, freqs_t, freqs_i):
        cfg = self.cfg
        b, si, _ = img.shape
        st = txt.shape[1]
        hl = cfg.heads // self.tp
        c = hl * cfg.head_dim
        sh1i, sc1i, g1i, sh2i, sc2i, g2i = self._mod_chunks(mod_i, b, cfg.hidden)
        sh1t, sc1t, g1t, sh2t, sc2t, g2t = self._mod_chunks(mod_t, b, cfg.hidden)
        ops = self.ops
        if hasattr(ops, "adaln_qkv_rope_into"):
            # q / k / v of [text; image] written by the projections into one
            # joint buffer that attention reads in place
            joint = torch.empty((b, st + si, 3 * c), dtype=torch.bfloat16, device=img.device)
            ops.adaln_qkv_rope_into(txt, sc1t, sh1t, bp.txt.qkv, bp.txt.qk_norm, freqs_t, 2 * c,
                                    [joint[i, :st] for i in range(b)], cfg.eps)
            ops.adaln_qkv_rope_into(img, sc1i, sh1i, bp.img.qkv, bp.img.qk_norm, freqs_i, 2 * c,
                                    [joint[i, st:] for i in range(b)], cfg.eps)
        else:
            qkv_i = ops.adaln_qkv_rope(img, sc1i, sh1i, bp.img.qkv, bp.img.qk_norm, freqs_i, 2 * c,
                                       cfg.eps)
            qkv_t = ops.adaln_qkv_rope(txt, sc1t, sh1t, bp.txt.qkv, bp.txt.qk_norm, freqs_t, 2 * c,
                                       cfg.eps)
            joint = torch.cat([qkv_t.reshape(b, st, 3 * c), qkv_i.reshape(b, si, 3 * c)], dim=1)
        o = ops.attention(joint, hl, cfg.head_dim)
        o_t, o_i = o[:, :st], o[:, st:]
        img = self._row_parallel(o_i, bp.img.out, img, g1i)
        txt = self._row_parallel(o_t, bp.txt.out, txt, g1t)
        h_i = ops.adaln_linear(img, sc2i, sh2i, bp.img.up, act="gelu_tanh", eps=cfg.eps)
        img = self._row_parallel(h_i, bp.img.down, img, g2i)
        h_t = ops.adaln_linear(txt, sc2t, sh2t, bp.txt.up, act="gelu_tanh", eps=cfg.eps)
        txt = self._row_parallel(h_t, bp.txt.down, txt, g2t)
        return img, txt

    def block_sp(self, bp: BlockParams, img, txt, mod_i, mod_t, freqs_t, freqs_i):
        """One joint block on a sequence-parallel rank: ``img`` [1, S/sp,
        hidden] is this rank's share of the image tokens (``freqs_i`` their
        rotations), ``txt`` all text tokens (every rank computes the text
        stream).  Each rank writes the k, v of its image tokens into its slot
        of the joint k / v buffer, one in-place all-gather fills the other
        slots, and its queries (all text tokens and its image tokens) attend
        to the whole sequence; every linear after that is row-local."""
        cfg, ops = self.cfg, self.ops
        b, sl, _ = img.shape
        if b != 1:
            raise ValueError("sequence parallelism runs one sample per call")
        st = txt.shape[1]
        c = cfg.hidden
        sh1i, sc1i, g1i, sh2i, sc2i, g2i = self._mod_chunks(mod_i, b, cfg.hidden)
        sh1t, sc1t, g1t, sh2t, sc2t, g2t = self._mod_chunks(mod_t, b, cfg.hidden)
        q = torch.empty((1, st + sl, c), dtype=torch.bfloat16, device=img.device)
        kv = torch.empty((1, st + sl * self.sp, 2 * c), dtype=torch.bfloat16, device=img.device)
        mine = kv[0, st + self.sp_rank * sl: st + (self.sp_rank + 1) * sl]
        ops.adaln_qkv_rope_split(txt, sc1t, sh1t, bp.txt.qkv, bp.txt.qk_norm, freqs_t,
                                 [q[0, :st]], [kv[0, :st]], cfg.eps)
        ops.adaln_qkv_rope_split(img, sc1i, sh1i, bp.img.qkv, bp.img.qk_norm, freqs_i,
                                 [q[0, st:]], [mine], cfg.eps)
        dist.all_gather_into_tensor(kv[0, st:], mine, group=self.sp_group)
        o = ops.attention_split(q, kv, cfg.heads, cfg.head_dim)
        img = ops.linear(o[:, st:], bp.img.out, residual=img, gate=g1i)
        txt = ops.linear(o[:, :st], bp.txt.out, residual=txt, gate=g1t)
        h_i = ops.adaln_linear(img, sc2i, sh2i, bp.img.up, act="gelu_tanh", eps=cfg.eps)
        img = ops.linear(h_i, bp.img.down, residual=img, gate=g2i)
        h_t = ops.adaln_linear(txt, sc2t, sh2t, bp.txt.up, act="gelu_tanh", eps=cfg.eps)
        txt = ops.linear(h_t, bp.txt.down, residual=txt, gate=g2t)
        return img, txt

    # -- the forward -------------------------------------------------------------
    def embed(self, latent, t, context):
        """Input projections and the modulation rows of every block."""
        cfg, p, ops = self.cfg, self.p, self.ops
        b, _, h, w = latent.shape
        img = patchify(latent.to(torch.bfloat16), cfg.patch)
        img = ops.linear(img, p.img_in)
        txt = ops.linear(context.to(torch.bfloat16), p.txt_in, input_norm=p.txt_norm, eps=cfg.eps)
        emb = timestep_embedding(round_timesteps(t).float(), cfg.time_dim).to(torch.bfloat16)
        temb = ops.linear(ops.silu(ops.linear(emb, p.time1)), p.time2)
        s = ops.silu(temb)
        mods_i = self._mod_linear(s, p.mod_img)
        mods_t = self._mod_linear(s, p.mod_txt)
        return img, txt, s, mods_i, mods_t

    def forward(self, latent: torch.Tensor, t: torch.Tensor, context: torch.Tensor,
                blocks: Optional[int] = None) -> torch.Tensor:
        """latent [B, C, H, W], t [B] (sigma in [0, 1]), context [B, S_txt,
        context_dim] -> the velocity prediction [B, C, H, W] (bf16)."""
        cfg, p, ops = self.cfg, self.p, self.ops
        b, c, h, w = latent.shape
        img, txt, s, mods_i, mods_t = self.embed(latent, t, context)
        freqs_t, freqs_i = self.freqs(txt.shape[1], h // cfg.patch, w // cfg.patch, latent.device)
        n = len(p.blocks) if blocks is None else blocks
        # every block's six modulation rows as contiguous [B, hidden] chunks
        # (one copy per stream and step): [blocks, 6, B, hidden]
        nb = mods_i.shape[1] // cfg.mod_dim
        mods_i = mods_i.reshape(b, nb, 6, cfg.hidden).permute(1, 2, 0, 3).contiguous()
        mods_t = mods_t.reshape(b, nb, 6, cfg.hidden).permute(1, 2, 0, 3).contiguous()
        block = self.block
        if self.sp > 1:
            # this rank's contiguous share of the image tokens
            mine = _shard(img.shape[1], self.sp_rank, self.sp)
            img = img[:, mine].contiguous()
            freqs_i = freqs_i[mine]
            block = self.block_sp
        for i, bp in enumerate(p.blocks[:n]):
            img, txt = block(bp, img, txt, mods_i[i], mods_t[i], freqs_t, freqs_i)
        scale, shift = ops.linear(s, p.norm_out).reshape(b, 2, 1, cfg.hidden).unbind(1)
        out = ops.adaln_linear(img, scale, shift, p.proj_out, eps=cfg.eps)
        if self.sp > 1:
            full = torch.empty((self.sp * out.shape[1], out.shape[2]), dtype=out.dtype,
                               device=out.device)
            dist.all_gather_into_tensor(full, out[0].contiguous(), group=self.sp_group)
            out = full.reshape(1, -1, out.shape[-1])
        return unpatchify(out, cfg.patch, c, h, w)


# --------------------------------------------------------------------------
# placement and the denoising step
# --------------------------------------------------------------------------
@dataclass
class Placement:
    """Where a CFG step runs: ``world`` ranks; one rank (both branches
    batched) or a branch per group of ``tp`` ranks (``tp`` is the group's
    width whatever its mode); this rank's branch and rank in the group;
    ``mode``: how a group of more than one rank splits its branch --
    "sequence" (image tokens split, whole weights) or "tensor" (heads and
    MLP columns split)."""
    world: int
    rank: int
    tp: int
    branch: int
    tp_rank: int
    mode: str = "sequence"

    @property
    def batched(self) -> bool:
        return self.world == 1

    @property
    def tensor_parallel(self) -> bool:
        return self.tp > 1 and self.mode == "tensor"

    @property
    def sequence_parallel(self) -> bool:
        return self.tp > 1 and self.mode == "sequence"

    def describe(self) -> str:
        if self.world == 1:
            return "1 GPU: both CFG branches batched (B = 2)"
        if self.tp == 1:
            return f"{self.world} GPUs: one CFG branch per GPU, predictions all-gathered"
        if self.mode == "sequence":
            return (f"{self.world} GPUs: CFG branch per group of {self.tp} GPUs, the image tokens "
                    f"split {self.tp} ways (whole weights; image k / v all-gathered per block, "
                    "text stream on every rank), predictions all-gathered")
        return (f"{self.world} GPUs: CFG branch per group of {self.tp} GPUs x {self.tp}-way tensor "
                "parallel (column-parallel QKV / MLP-up, row-parallel out / MLP-down with exact "
                "int32 reductions), predictions all-gathered")


def placement(world: int, rank: int, mode: str = "sequence") -> Placement:
    """1 rank: both branches batched.  W >= 2 (even): ranks [0, W/2) run the
    conditional branch, [W/2, W) the unconditional one, each branch over W/2
    ranks split by ``mode`` ("sequence" or "tensor")."""
    if mode not in ("sequence", "tensor"):
        raise ValueError(f"unknown placement mode {mode!r}")
    if world == 1:
        return Placement(1, 0, 1, 0, 0, mode)
    if world % 2:
        raise ValueError("CFG placement needs an even number of ranks")
    tp = world // 2
    return Placement(world, rank, tp, rank // tp, rank % tp, mode)


class ProcessGroups:
    """The group of this rank's branch (``tp_group``, tensor- or
    sequence-parallel) and the CFG pair group (r, r + W/2); every rank
    creates every group in the same order."""

    def __init__(self, pl: Placement, backend=None):
        self.tp_group = None
        self.cfg_group = None
        if pl.world == 1:
            return
        for br in range(2):
            ranks = list(range(br * pl.tp, (br + 1) * pl.tp))
            g = dist.new_group(ranks, backend=backend) if pl.tp > 1 else None
            if br == pl.branch:
                self.tp_group = g
        for r in range(pl.tp):
            g = dist.new_group([r, r + pl.tp], backend=backend)
            if r == pl.tp_rank:
                self.cfg_group = g


def build_model(cfg: MMDiTConfig, ops, device, pl: Placement, groups: ProcessGroups,
                seed: int = 0, fused_tp: bool = False) -> MMDiT:
    """Random-init weights and the model of this rank for ``pl``."""
    if pl.tensor_parallel:
        params = random_params(cfg, ops, device, seed=seed, tp_rank=pl.tp_rank, tp_world=pl.tp)
        return MMDiT(params, ops, groups.tp_group, fused_tp=fused_tp)
    params = random_params(cfg, ops, device, seed=seed)
    return MMDiT(params, ops, sp_group=groups.tp_group if pl.sequence_parallel else None)


def cfg_model(dit: MMDiT, pl: Placement, groups: ProcessGroups, context_cond: torch.Tensor,
              context_uncond: torch.Tensor):
    """The sampler's ``Model`` (imagine_b200.sampler): ``model(x, timestep,
    with_uncond)`` -> (conditional, unconditional) predictions.  On one GPU
    the branches run as one batch of 2 (the reference's batched CFG,
    inference/src/models/qwen_image21/cfg.rs:136-207); on 2+ GPUs each rank
    group runs its branch and the pair all-gather exchanges the outputs."""

    def model(x, timestep, with_uncond):
        xb = x.to(torch.bfloat16)
        if not with_uncond:
            return dit.forward(xb, timestep, context_cond), None
        if pl.batched:
            out = dit.forward(torch.cat([xb, xb]), torch.cat([timestep, timestep]),
                              torch.cat([context_cond, context_uncond]))
            n = x.shape[0]
            return out[:n], out[n:]
        ctx = context_cond if pl.branch == 0 else context_uncond
        mine = dit.forward(xb, timestep, ctx).contiguous()
        both = [torch.empty_like(mine), torch.empty_like(mine)]
        dist.all_gather(both, mine, group=groups.cfg_group)
        return both[0], both[1]

    return model


class CapturedModel:
    """``cfg_model`` replayed from one CUDA graph per call: the whole forward
    of both CFG branches (every block's kernels and, across GPUs, its NCCL
    collectives) is captured once and replayed, so a step costs one graph
    launch on the host instead of ~40 launches per block.  Inputs are copied
    into static buffers; the returned predictions are static buffers too,
    valid until the next call.  The fused peer-memory reductions number their
    exchanges on the host and cannot be replayed; a model built with
    ``fused_tp`` is refused."""

    def __init__(self, dit: MMDiT, pl: Placement, groups: ProcessGroups,
                 context_cond: torch.Tensor, context_uncond: torch.Tensor, x_shape, device):
        if dit.fused_tp:
            raise ValueError("the fused tensor-parallel reductions cannot be replayed from a graph")
        self.fn = cfg_model(dit, pl, groups, context_cond, context_uncond)
        self.x = torch.zeros(x_shape, dtype=torch.float32, device=device)
        self.t = torch.full((x_shape[0],), 0.5, dtype=torch.float32, device=device)
        self.graph = None
        self.out = None

    def capture(self, warmup: int = 2) -> None:
        side = torch.cuda.Stream(self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.fn(self.x, self.t, True)
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        torch.cuda.synchronize(self.x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self.fn(self.x, self.t, True)
        torch.cuda.synchronize(self.x.device)

    def __call__(self, x, timestep, with_uncond):
        if not with_uncond:
            raise ValueError("the captured model runs both CFG branches")
        if self.graph is None:
            self.capture()
        self.x.copy_(x)
        self.t.copy_(timestep)
        self.graph.replay()
        return self.out

    def release(self) -> None:
        """Drop the graph (and the collectives it holds) before the process
        group is destroyed."""
        self.graph = None
        self.out = None


class DenoiseLoop:
    """The Euler CFG loop of the sampler (inference/src/models/qwen_image21/
    sampling.rs:231-277) around ``cfg_model``, one step at a time:
    ``step(i)`` runs the model on both branches and the fused sampler step
    (imagine_b200.sampler) on the latent ``x``."""

    def __init__(self, model, x: torch.Tensor, steps: int = 40, cfg_scale: float = 2.5,
                 shift: float = 0.69):
        from . import sampler as S

        self.S = S
        self.model = model
        self.x = x.to(torch.float32).contiguous().clone()
        self.cfg_scale = cfg_scale
        sigmas = S.FluxSampling(shift).simple(steps).to(self.x.device)
        self.rows = [r for _, _, r in S.euler_coefficients(sigmas)]
        self.s_in = torch.ones(self.x.shape[0], dtype=torch.float32, device=self.x.device)

    def step(self, i: int) -> None:
        row = self.rows[i % len(self.rows)]
        out_c, out_u = self.model(self.x, row[0].mul(self.s_in), True)
        self.S.sampler_step(self.x, out_c.contiguous(), out_u.contiguous(), row,
                            self.S.N.STEP_EULER, cfg_scale=self.cfg_scale)
