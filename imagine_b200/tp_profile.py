"""Time the column-parallel W8A8 linear on N GPUs (one process per GPU, under
torchrun): the GEMM followed by an NCCL all-gather, against the GEMM whose
epilogue writes every output chunk into all ranks' outputs over NVLink.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \\
        --master-addr 127.0.0.1 --master-port 29500 -m imagine_b200.tp_profile

Seeded synthetic inputs of the MLP-up shape (5600 x 3072 -> 12288, GELU);
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
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
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


if __name__ == "__main__":
    main()
