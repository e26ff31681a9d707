"""Run one W8A8 kernel on one shape a few times -- the command the committed
ncu summaries under profiles/ were captured with.

    python -m imagine_b200.profile_case --kernel gemm --m 5600 --k 3072 --n 3072
    python -m imagine_b200.profile_case --kernel quantize --m 5600 --k 3072
    python -m imagine_b200.profile_case --kernel gemv --m 2 --k 3072 --n 18432

Inputs are seeded synthetic tensors of the BASELINE distributions; every
launch is checked for device errors afterwards.
"""
from __future__ import annotations

import argparse

import torch

import imagine_b200 as W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=["gemm", "gemm_gelu", "quantize", "gemv", "fp8_gemm"],
                    required=True)
    ap.add_argument("--m", type=int, default=5600)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--block-n", type=int, default=0)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(a.m, a.k, generator=g).to(torch.bfloat16).to(dev)
    cfg = (a.block_n, 8, 0)
    if a.kernel == "quantize":
        for _ in range(a.iters):
            W.quantize_int8_rowwise(x)
    else:
        w = (torch.randn(a.n, a.k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        b = (torch.randn(a.n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        wq, ws = W.quantize_weight(w)
        if a.kernel in ("gemm", "gemm_gelu", "gemv"):
            act = "gelu_tanh" if a.kernel == "gemm_gelu" else None
            for _ in range(a.iters):
                W.int8_linear(x, wq, ws, b, output_act=act, config=cfg)
        else:
            sa = (x.abs().max().float() / 448).reshape(1)
            sw = (w.abs().max().float() / 448).reshape(1)
            aq = W.quantize_per_tensor_fp8(x, sa)
            wq8 = W.quantize_per_tensor_fp8(w, sw)
            for _ in range(a.iters):
                W.fp8_linear(aq, sa, wq8, sw, b, config=cfg)
    torch.cuda.synchronize()
    err = W.device_error()
    if err:
        raise SystemExit(f"device error {err}")
    print("ok", a.kernel, a.m, a.k, a.n)


if __name__ == "__main__":
    main()
