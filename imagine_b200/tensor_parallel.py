"""Multi-GPU placement of the W8A8 linear family (one process per GPU).

The reference runs on a single GPU (design-document.md:92); this module adds
the two tensor-parallel forms of its `int8_linear` operator and the CFG/seed
placement plan.  Both linears are bit-identical to the single-GPU operator:

* ``ColumnParallelInt8Linear`` shards W along N.  Every rank quantises the full
  activation (identical codes on every rank), computes its N-slice, and
  optionally all-gathers the slices.  Used for QKV, MLP-up and the AdaLN
  modulation GEMV.  With ``fused=True`` the all-gather is not a collective
  after the GEMM: the GEMM's epilogue copies every finished output chunk into
  every peer's receive buffer over NVLink (w8a8_gemm_dequant_allgather), which
  every rank maps (torch's symmetric memory, used as plumbing), and each rank
  then places its peers' chunks (w8a8_allgather_finish).
* ``RowParallelInt8Linear`` shards W and the activation along K.  The per-token
  scale needs the absmax of the whole row, so ranks all-reduce(MAX) their
  shard's row absmax first; each rank then quantises its shard with the full
  row's scale (its codes equal the single-GPU codes of those columns), runs an
  int32 GEMM on its K-slice, and the int32 partial sums are all-reduced (SUM,
  exact) before one dequant epilogue.  Used for the out-projection and
  MLP-down.

The numeric steps are delegated to a backend object; ``NativeBackend`` is the
libw8a8 C ABI.  Collectives go through ``torch.distributed`` (NCCL on GPUs).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


class NativeBackend:
    """libw8a8 kernels (imagine_b200.linear)."""

    def __init__(self):
        from . import linear

        self.L = linear

    def linear(self, x, w, ws, bias, out_dtype, **kw):
        return self.L.int8_linear(x, w, ws, bias, out_dtype=out_dtype, **kw)

    def row_absmax(self, x):
        return self.L.row_absmax(x)

    def quantize_given_absmax(self, x, amax, scale_mode="eager"):
        return self.L.quantize_int8_rowwise_given_absmax(x, amax, scale_mode=scale_mode)

    def gemm_s32(self, q, w):
        return self.L.int8_gemm_s32(q, w)

    def dequant(self, acc, xs, ws, bias, out_dtype, dequant="eager"):
        return self.L.dequantize_int8_linear(acc, xs, ws, bias, out_dtype, dequant=dequant)


def split_sizes(total: int, world: int) -> List[int]:
    """Contiguous near-equal split (the first `total % world` ranks get one more)."""
    base, extra = divmod(total, world)
    return [base + (1 if r < extra else 0) for r in range(world)]


def shard_slice(total: int, rank: int, world: int) -> slice:
    sizes = split_sizes(total, world)
    start = sum(sizes[:rank])
    return slice(start, start + sizes[rank])


class _PeerBuffers:
    """Peer-mapped receive buffer and flag block of one fused column-parallel
    linear, on every rank of `group` (rendezvous is collective: every rank
    makes the same calls in the same order)."""

    def __init__(self, group, device):
        import torch.distributed._symmetric_memory as symm

        from . import _native as N

        self.symm = symm
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.flags = symm.empty(N.PEER_FLAG_WORDS, dtype=torch.int32, device=device)
        self.flags.zero_()
        handle = symm.rendezvous(self.flags, self.group)
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*handle.buffer_ptrs)
        self._keep = [handle]
        self.recv_ptrs = None
        self.epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(self.group)  # every flag block is zero before any rank signals

    def _mapped(self, attr: str, nbytes: int, device):
        """A peer-mapped byte buffer of at least `nbytes` under `attr`, and the
        array of every rank's pointer to it (collective on first use and on
        growth)."""
        cur = getattr(self, attr, None)
        if cur is None or cur[0].numel() < nbytes:
            # a peer may still be writing into the old buffer: finish first
            torch.cuda.synchronize(device)
            dist.barrier(self.group)
            buf = self.symm.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
            handle = self.symm.rendezvous(buf, self.group)
            ptrs = (ctypes.c_void_p * self.world)(*handle.buffer_ptrs)
            self._keep.append((buf, handle))
            setattr(self, attr, (buf, ptrs))
        return getattr(self, attr)[1]

    def receive(self, nbytes: int, device) -> None:
        self.recv_ptrs = self._mapped("_recv", nbytes, device)

    def next_epoch(self) -> int:
        self.epoch = self.epoch % 0xFFFFFFFF + 1  # never 0
        return self.epoch


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


class ColumnParallelInt8Linear:
    """W [N, K] int8 sharded along N; y = x W^T with each rank owning an N slice."""

    def __init__(self, weight: torch.Tensor, weight_scale: torch.Tensor,
                 bias: Optional[torch.Tensor] = None, *, group=None, gather_output: bool = True,
                 backend=None, fused: bool = False, **linear_kwargs):
        self.group = group
        self.rank, self.world = _world(group)
        n = weight.shape[0]
        self.n = n
        sl = shard_slice(n, self.rank, self.world)
        self.col_offset = sl.start
        self.sizes = split_sizes(n, self.world)
        self.weight = weight[sl].contiguous()
        ws = weight_scale.reshape(-1)
        self.weight_scale = ws if ws.numel() == 1 else ws[sl].contiguous()
        self.bias = bias[sl].contiguous() if bias is not None else None
        self.gather_output = gather_output
        self.backend = backend or NativeBackend()
        self.kw = linear_kwargs
        self.fused = (fused and gather_output and self.world > 1 and
                      len(set(self.sizes)) == 1 and self.sizes[0] % 8 == 0 and
                      set(linear_kwargs) <= {"dequant", "scale_mode", "output_act"})
        self._peers = None

    def _fused_call(self, x: torch.Tensor, out_dtype) -> torch.Tensor:
        """Quantise x, then the GEMM whose epilogue also sends this rank's
        chunks to every peer, then this rank's copy of the peers' chunks (see
        the module doc)."""
        from . import _native as N
        from .linear import _code, _epilogue, _stream, _vp, quantize_int8_rowwise

        dev = x.device
        if self._peers is None:
            self._peers = _PeerBuffers(self.group, dev)
        pb = self._peers
        lead = x.shape[:-1]
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        m = x2.shape[0]
        ns = self.weight.shape[0]
        y = torch.empty((m, self.n), dtype=out_dtype, device=dev)
        if m == 0:
            return y.reshape(*lead, self.n)
        pb.receive(int(N.LIB.w8a8_allgather_recv_bytes(m, ns, _code(out_dtype), self.world)), dev)
        epoch = pb.next_epoch()
        stream = _stream(dev)
        N.check(N.LIB.w8a8_peer_barrier(pb.flag_ptrs, self.rank, self.world, epoch, stream))
        q, xs = quantize_int8_rowwise(x2, scale_mode=self.kw.get("scale_mode", "eager"))
        ws = self.weight_scale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        b = self.bias.to(device=dev, dtype=out_dtype).contiguous() if self.bias is not None else None
        ep = _epilogue(ws, b, None, None, self.kw.get("dequant", "eager"),
                       self.kw.get("output_act"), ns, ns)
        N.check(N.LIB.w8a8_gemm_dequant_allgather(
            _vp(q), k, _vp(self.weight), k, _vp(xs.reshape(-1)), ctypes.byref(ep), _vp(y),
            _code(out_dtype), self.n, m, ns, k, pb.recv_ptrs, pb.flag_ptrs, self.rank, self.world,
            epoch, None, stream))
        N.check(N.LIB.w8a8_allgather_finish(_vp(y), _code(out_dtype), self.n, m, ns, pb.recv_ptrs,
                                            pb.flag_ptrs, self.rank, self.world, epoch, stream))
        return y.reshape(*lead, self.n)

    def __call__(self, x: torch.Tensor, out_dtype=None) -> torch.Tensor:
        if self.fused:
            return self._fused_call(x, out_dtype or x.dtype)
        y = self.backend.linear(x, self.weight, self.weight_scale, self.bias,
                                out_dtype or x.dtype, **self.kw)
        if not self.gather_output or self.world == 1:
            return y
        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        parts = [torch.empty((y2.shape[0], s), dtype=y2.dtype, device=y2.device) for s in self.sizes]
        if len(set(self.sizes)) == 1:
            dist.all_gather(parts, y2, group=self.group)
        else:  # uneven shards: gather padded rows, then trim
            pad = max(self.sizes)
            buf = torch.zeros((y2.shape[0], pad), dtype=y2.dtype, device=y2.device)
            buf[:, : y2.shape[1]] = y2
            padded = [torch.empty_like(buf) for _ in self.sizes]
            dist.all_gather(padded, buf, group=self.group)
            parts = [p[:, :s] for p, s in zip(padded, self.sizes)]
        return torch.cat(parts, dim=-1).reshape(*lead, -1)


class RowParallelInt8Linear:
    """W [N, K] int8 sharded along K; the input arrives sharded along K.

    Each rank quantises its K-slice with the full rows' scales (an all-reduce
    MAX of the per-row absmax) and computes an exact int32 partial product.
    With ``fused=False`` an NCCL all-reduce SUM of the partials follows, then
    the dequant epilogue.  With ``fused=True`` the reduction is no collective
    after the GEMM: the GEMM's epilogue sends every finished int32 partial
    chunk to the rank that owns its rows (w8a8_gemm_s32_reduce_scatter), and
    each rank sums its rows, applies the epilogue and hands its rows to the
    others (w8a8_reduce_scatter_finish), over buffers every rank maps (torch's
    symmetric memory, used as plumbing).  Both equal the single-GPU linear bit
    for bit."""

    def __init__(self, weight: torch.Tensor, weight_scale: torch.Tensor,
                 bias: Optional[torch.Tensor] = None, *, group=None, backend=None,
                 dequant: str = "eager", scale_mode: str = "eager", fused: bool = False):
        self.group = group
        self.rank, self.world = _world(group)
        k = weight.shape[1]
        self.k_slice = shard_slice(k, self.rank, self.world)
        self.weight = weight[:, self.k_slice].contiguous()
        self.weight_scale = weight_scale.reshape(-1)
        self.bias = bias
        self.backend = backend or NativeBackend()
        self.dequant = dequant
        self.scale_mode = scale_mode
        self.fused = (fused and self.world > 1 and weight.shape[0] % 8 == 0
                      and isinstance(self.backend, NativeBackend))
        self._peers = None

    def shard_input(self, x_full: torch.Tensor) -> torch.Tensor:
        return x_full[..., self.k_slice].contiguous()

    def __call__(self, x_shard: torch.Tensor, out_dtype=None) -> torch.Tensor:
        out_dtype = out_dtype or x_shard.dtype
        lead = x_shard.shape[:-1]
        x2 = x_shard.reshape(-1, x_shard.shape[-1])
        amax = self.backend.row_absmax(x2).reshape(-1).contiguous()
        if self.world > 1:
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        q, xs = self.backend.quantize_given_absmax(x2, amax, scale_mode=self.scale_mode)
        if self.fused and x2.shape[0] > 0:
            return self._fused_call(q, xs, out_dtype).reshape(*lead, -1)
        acc = self.backend.gemm_s32(q, self.weight)
        if self.world > 1:
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        y = self.backend.dequant(acc, xs, self.weight_scale, self.bias, out_dtype, dequant=self.dequant)
        return y.reshape(*lead, -1)

    def _fused_call(self, q: torch.Tensor, xs: torch.Tensor, out_dtype) -> torch.Tensor:
        """The GEMM with the reduce-scatter in its epilogue, then the finish (see
        the class doc).  The ready barrier comes first so that no rank writes
        into a peer's buffers before that peer has consumed the previous
        call's."""
        from . import _native as N
        from .linear import _code, _epilogue, _stream, _vp

        dev = q.device
        m, k = q.shape
        n = self.weight.shape[0]
        if self._peers is None:
            self._peers = _PeerBuffers(self.group, dev)
        pb = self._peers
        recvs = pb._mapped("_rs_recv", int(N.LIB.w8a8_reduce_scatter_recv_bytes(m, n, self.world)),
                           dev)
        esz = torch.empty((), dtype=out_dtype).element_size()
        stages = pb._mapped("_rs_stage", m * n * esz, dev)
        y = torch.empty((m, n), dtype=out_dtype, device=dev)
        epoch = pb.next_epoch()
        stream = _stream(dev)
        N.check(N.LIB.w8a8_peer_barrier(pb.flag_ptrs, self.rank, self.world, epoch, stream))
        N.check(N.LIB.w8a8_gemm_s32_reduce_scatter(_vp(q), k, _vp(self.weight), k, m, n, k, recvs,
                                                   pb.flag_ptrs, self.rank, self.world, epoch,
                                                   None, stream))
        ws = self.weight_scale.to(device=dev, dtype=torch.float32).contiguous()
        b = self.bias.to(device=dev, dtype=out_dtype).contiguous() if self.bias is not None else None
        ep = _epilogue(ws, b, None, None, self.dequant, None, n, n)
        N.check(N.LIB.w8a8_reduce_scatter_finish(_vp(xs.reshape(-1)), ctypes.byref(ep), _vp(y),
                                                 _code(out_dtype), n, m, n, recvs, stages,
                                                 pb.flag_ptrs, self.rank, self.world, epoch,
                                                 stream))
        return y


def cfg_placement(world: int, samples: int, branches: int = 2) -> List[List[Tuple[int, int]]]:
    """Which (sample, branch) units each rank runs: unit u = sample * branches +
    branch goes to rank u % world (GPU g runs branch g mod 2 of sample g // 2
    when world = 2 * samples).  Units are independent until the CFG combine."""
    plan: List[List[Tuple[int, int]]] = [[] for _ in range(world)]
    for u in range(samples * branches):
        plan[u % world].append((u // branches, u % branches))
    return plan
