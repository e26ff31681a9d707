"""Time the tensor-parallel W8A8 linears on N GPUs (one process per GPU, under
torchrun).  Column-parallel (default): the GEMM followed by an NCCL
all-gather, against the GEMM whose epilogue copies every output chunk to all
ranks over NVLink.  Row-parallel (``--row``): the int32 partial GEMM followed
by an NCCL all-reduce and the dequant, against the GEMM whose epilogue sends
each partial chunk to the rank owning its rows plus the fused finish.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \\
        --master-addr 127.0.0.1 --master-port 29500 -m imagine_b200.tp_profile [--row]

Seeded synthetic inputs of the MLP-up shape (5600 x 3072 -> 12288, GELU) or,
with --row, of the MLP-down shape (5600 x 12288 -> 3072);
each form runs W untimed then K timed calls, L2 flushed before each; the time
is the max over ranks of the per-call CUDA-event time on the launching stream.
Prints one JSON line (rank 0)."""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=5600)
    ap.add_argument("--k", type=int, default=None)
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--row", action="store_true", help="row-parallel (K-sharded) linear")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    a.k = a.k or (12288 if a.row else 3072)
    a.n = a.n or (3072 if a.row else 12288)
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    world = dist.get_world_size()

    import imagine_b200 as W
    from imagine_b200 import tensor_parallel as TP

    g = torch.Generator().manual_seed(0)
    x = torch.randn(a.m, a.k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(a.n, a.k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    b = (torch.randn(a.n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wq, ws = W.quantize_weight(w)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    clean = torch.ones_like(flush)
    if a.row:
        return _row(a, rank, world, dev, x, wq, ws, b, flush, clean)
    forms = {"nccl_all_gather": TP.ColumnParallelInt8Linear(wq, ws, b, output_act="gelu_tanh"),
             "fused_peer_stores": TP.ColumnParallelInt8Linear(wq, ws, b, output_act="gelu_tanh",
                                                              fused=True),
             "local_shard_only": TP.ColumnParallelInt8Linear(wq, ws, b, output_act="gelu_tanh",
                                                             gather_output=False)}
    local = forms["local_shard_only"]

    class _IntoTensor:
        """GEMM, then NCCL's all_gather_into_tensor and one transposing copy
        into [M, N]: the fastest NCCL form of the same exchange."""

        def __call__(self, xi):
            y = local(xi)
            buf = torch.empty((world,) + tuple(y.shape), dtype=y.dtype, device=y.device)
            dist.all_gather_into_tensor(buf, y.contiguous())
            return buf.permute(1, 0, 2).reshape(y.shape[0], -1)

    if len(set(TP.split_sizes(a.n, world))) == 1:
        forms["nccl_all_gather_into_tensor"] = _IntoTensor()
    ref = W.int8_linear(x, wq, ws, b, output_act="gelu_tanh")
    out = {}
    for name, layer in forms.items():
        for _ in range(a.warmup):
            layer(x)
        torch.cuda.synchronize()
        times = []
        for _ in range(a.steps):
            flush.zero_()
            clean.sum()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            y = layer(x)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        t = torch.tensor(sorted(times)[len(times) // 2], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        exact = name == "local_shard_only" or torch.equal(y.view(torch.int16), ref.view(torch.int16))
        ok = torch.tensor(int(exact), device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        out[name] = {"ms": float(t), "bit_exact_vs_1gpu": bool(ok)}
    if W.device_error() != 0:
        raise RuntimeError("device error")
    if rank == 0:
        ops = 2.0 * a.m * a.n * a.k
        for v in out.values():
            v["TOPS"] = ops / (v["ms"] * 1e-3) / 1e12
        print(json.dumps({"workload": "column-parallel int8 linear + GELU", "M": a.m, "K": a.k,
                          "N": a.n, "world": world, "forms": out,
                          "gather_bytes_per_rank": a.m * (a.n - a.n // world) * 2}))
    forms.clear()
    dist.destroy_process_group()


def _row(a, rank, world, dev, x, wq, ws, b, flush, clean):
    import imagine_b200 as W
    from imagine_b200 import _native
    from imagine_b200 import tensor_parallel as TP

    nccl = TP.RowParallelInt8Linear(wq, ws, b)
    fused = TP.RowParallelInt8Linear(wq, ws, b, fused=True)
    assert fused.fused
    x_shard = nccl.shard_input(x)
    be = nccl.backend

    def partial_only(xi):
        """Quantise (with the all-reduce MAX of the row absmax) and the int32
        partial GEMM: no exchange of the partials, no dequant."""
        amax = be.row_absmax(xi).reshape(-1).contiguous()
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        q, _ = be.quantize_given_absmax(xi, amax)
        return be.gemm_s32(q, nccl.weight)

    ref = W.int8_linear(x, wq, ws, b)
    out = {}
    for name, layer in (("nccl_all_reduce", nccl), ("fused_reduce_scatter", fused),
                        ("local_partial_only", partial_only)):
        for _ in range(a.warmup):
            layer(x_shard)
        torch.cuda.synchronize()
        times = []
        for _ in range(a.steps):
            flush.zero_()
            clean.sum()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            y = layer(x_shard)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        t = torch.tensor(sorted(times)[len(times) // 2], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        exact = name == "local_partial_only" or torch.equal(y.view(torch.int16), ref.view(torch.int16))
        ok = torch.tensor(int(exact), device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        out[name] = {"ms": float(t), "bit_exact_vs_1gpu": bool(ok)}
    if W.device_error() != 0:
        raise RuntimeError("device error")
    if rank == 0:
        ops = 2.0 * a.m * a.n * a.k
        for v in out.values():
            v["TOPS"] = ops / (v["ms"] * 1e-3) / 1e12
        rows = int(_native.LIB.w8a8_reduce_scatter_rows(a.m, world))
        print(json.dumps({"workload": "row-parallel int8 linear", "M": a.m, "K": a.k, "N": a.n,
                          "world": world, "forms": out,
                          "partial_bytes_sent_by_rank0": (a.m - min(a.m, rows)) * a.n * 4}))
    del fused
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
