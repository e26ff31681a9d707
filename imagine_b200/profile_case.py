"""Run one W8A8 kernel on one shape a few times -- the command the committed
ncu summaries under profiles/ were captured with.

    python -m imagine_b200.profile_case --kernel gemm --m 5600 --k 3072 --n 3072
    python -m imagine_b200.profile_case --kernel quantize --m 5600 --k 3072
    python -m imagine_b200.profile_case --kernel gemv --m 2 --k 3072 --n 18432
    python -m imagine_b200.profile_case --kernel gemm_rope --m 5600 --k 3072 --n 9216 --rope-cols 6144
    python -m imagine_b200.profile_case --kernel compare_libraries --iters 20

``compare_libraries`` times, on the same device buffers, this library's
INT8 / FP8 / MXFP8 GEMMs against the library kernels the reference's sm_100
routes call: cuBLASLt INT8 through torch._int_mm (the reference's
``cublas_gemm_int8``, KSRC backends/cuda/ops/cublas_gemm_int8.cu:89-230, then
its separate dequant), cuBLASLt FP8 TensorWise through torch._scaled_mm
(``imagine_fp8_scaled_mm``, inference/native/bridge.cpp:401-413) and cuBLASLt
MXFP8 with e8m0 block scales through torch._scaled_mm (``scaled_mm_mxfp8``,
inference/src/backend_quant.rs:320-343), at 5600 x 3072 -> 12288 and -> 3072.
It prints one JSON line.

Inputs are seeded synthetic tensors of the BASELINE distributions; every
launch is checked for device errors afterwards.
"""
from __future__ import annotations

import argparse

import torch

import imagine_b200 as W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=["gemm", "gemm_gelu", "gemm_s32", "quantize", "convrot",
                                                       "gemv", "fp8_gemm", "mxfp8_gemm", "rms_rope",
                                                       "gemm_rope", "sampler_euler", "sampler_er_sde", "gemv_q",
                                                       "compare_libraries", "modulated", "dit_step"],
                    required=True)
    ap.add_argument("--m", type=int, default=5600)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--block-n", type=int, default=0)
    ap.add_argument("--cta-group", type=int, default=0)
    ap.add_argument("--rope-cols", type=int, default=-1,
                    help="gemm_rope: columns that get RMSNorm + RoPE (default: all)")
    ap.add_argument("--tiled", action="store_true", help="GEMM on the pre-tiled weight layout")
    ap.add_argument("--split-k", type=int, default=1,
                    help="GEMM K splits (0: chosen from the SM count, 1: off)")
    ap.add_argument("--mode", default="adaln",
                    choices=["scale", "rms_scale", "adaln", "rms_adaln"],
                    help="modulated: the modulation fused into the quantiser (rows of --m split "
                         "into two samples)")
    ap.add_argument("--blocks", type=int, default=60, help="dit_step: MMDiT blocks")
    ap.add_argument("--time", action="store_true",
                    help="time each launch with CUDA events (L2 flushed before each) and print "
                         "the median")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(a.m, a.k, generator=g).to(torch.bfloat16).to(dev)
    cfg = (a.block_n, 8, 0, a.cta_group)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev) if a.time else None
    clean = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev) if a.time else None
    times = []

    def run(fn):
        for _ in range(a.iters):
            if flush is not None:
                # a ~100 us GPU sleep first gives the host time to enqueue the
                # flush, the events and the launch, so no host work lands inside
                # the timed window; the flush writes 256 MiB and reads another
                # 256 MiB (cold L2 with no dirty lines left by the flush)
                torch.cuda._sleep(200000)
                flush.zero_()
                clean.sum()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            else:
                fn()

    if a.kernel == "compare_libraries":
        return compare_libraries(a, dev, g, flush, clean)
    if a.kernel == "dit_step":
        # --iters eager denoising steps of the MMDiT at 1600x896, both CFG
        # branches batched on this GPU (the launch list of one step: skip the
        # set-up and warm-up launches, capture about 25 x --blocks launches)
        from imagine_b200 import mmdit as MD

        cfg_m = MD.MMDiTConfig(blocks=a.blocks)
        ops = MD.NativeOps()
        pl = MD.placement(1, 0)
        groups = MD.ProcessGroups(pl)
        dit = MD.build_model(cfg_m, ops, dev, pl, groups, seed=1)
        lat = torch.randn(1, 16, 112, 200, generator=g).to(dev)
        cc = torch.randn(1, 256, 3072, generator=g).to(torch.bfloat16).to(dev)
        cu = torch.randn(1, 256, 3072, generator=g).to(torch.bfloat16).to(dev)
        loop = MD.DenoiseLoop(MD.cfg_model(dit, pl, groups, cc, cu), lat)
        step = [0]

        def one():
            # every step after the first inside the NVTX range "dit_step" (for
            # ncu --nvtx --nvtx-include dit_step/)
            if step[0]:
                torch.cuda.nvtx.range_push("dit_step")
            loop.step(step[0])
            if step[0]:
                torch.cuda.nvtx.range_pop()
            step[0] += 1
        run(one)
        a.m, a.k, a.n = 1, 1, 1
    elif a.kernel == "modulated":
        b2 = 2 if a.m % 2 == 0 else 1
        xm = x.reshape(b2, a.m // b2, a.k)
        sc = (0.3 * torch.randn(b2, 1, a.k, generator=g)).to(torch.bfloat16).to(dev)
        sh = (0.3 * torch.randn(b2, 1, a.k, generator=g)).to(torch.bfloat16).to(dev)
        nw = (1 + 0.1 * torch.randn(a.k, generator=g)).to(torch.bfloat16).to(dev)
        if a.mode in ("scale", "rms_scale"):
            sc = sc[:1]
        run(lambda: W.quantize_int8_rowwise_modulated(
            xm, a.mode, sc, sh if "adaln" in a.mode else None,
            nw if a.mode == "rms_scale" else None))
    elif a.kernel.startswith("sampler_"):
        # one fused sampler step over an fp32 latent of --m x --k elements with
        # bf16 branch outputs (ER-SDE: stage 3 with noise)
        from imagine_b200 import _native as NAT
        from imagine_b200 import sampler as SM
        shape = (a.m, a.k)
        lat = torch.randn(shape, generator=g).to(dev)
        oc = torch.randn(shape, generator=g).to(torch.bfloat16).to(dev)
        ou = torch.randn(shape, generator=g).to(torch.bfloat16).to(dev)
        coef = (torch.rand(9, generator=g) + 0.5).to(dev)
        if a.kernel == "sampler_euler":
            run(lambda: SM.sampler_step(lat, oc, ou, coef, NAT.STEP_EULER, cfg_scale=2.5))
        else:
            od, odr = torch.zeros_like(lat), torch.zeros_like(lat)
            nz = torch.randn(shape, generator=g).to(dev)
            run(lambda: SM.sampler_step(lat, oc, ou, coef, NAT.STEP_ER_SDE, cfg_scale=2.5, stage=3,
                                        old_denoised=od, old_derivative=odr, noise=nz))
    elif a.kernel == "quantize":
        run(lambda: W.quantize_int8_rowwise(x))
    elif a.kernel == "convrot":
        run(lambda: W.quantize_int8_rowwise_convrot(x, 256))
    elif a.kernel == "rms_rope":
        # q and k of m tokens with k / 128 heads of 128
        heads = a.k // 128
        kk = torch.randn(a.m, a.k, generator=g).to(torch.bfloat16).to(dev)
        ang = torch.rand(a.m, 64, generator=g) * 6.283
        c, sn = torch.cos(ang), torch.sin(ang)
        f = torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2).to(dev)
        sc = torch.ones(128, dtype=torch.bfloat16, device=dev)
        qv, kv = x.view(a.m, heads, 128), kk.view(a.m, heads, 128)
        run(lambda: W.rms_rope(qv, kv, f, sc, sc, 1e-6))
    else:
        w = (torch.randn(a.n, a.k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        b = (torch.randn(a.n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        wq, ws = W.quantize_weight(w)
        if a.kernel == "gemm_rope":
            # the projection with its RMSNorm + RoPE epilogue, on pre-quantised
            # activations (rows are the tokens of one sequence)
            import ctypes
            from imagine_b200 import _native as NAT
            from imagine_b200.linear import _config, _epilogue, _stream, _vp
            rc = a.n if a.rope_cols < 0 else a.rope_cols
            q, xs = W.quantize_int8_rowwise(x)
            y = torch.empty((a.m, a.n), dtype=torch.bfloat16, device=dev)
            ep = _epilogue(ws, b, None, None, "eager", None, a.n, a.n)
            c = _config(cfg)
            ang = torch.rand(a.m, 64, generator=g) * 6.283
            cs, sn = torch.cos(ang), torch.sin(ang)
            f = torch.stack([torch.stack([cs, -sn], -1), torch.stack([sn, cs], -1)], -2).to(dev)
            nw = torch.ones(max(rc, 128), dtype=torch.bfloat16, device=dev)
            nbytes = 0
            if a.split_k == 0:
                with torch.cuda.device(dev):
                    nbytes = NAT.LIB.w8a8_gemm_auto_workspace_bytes(a.m, a.n, a.k, ctypes.byref(c))
            elif a.split_k > 1:
                nbytes = NAT.LIB.w8a8_gemm_splitk_workspace_bytes(a.m, a.n)
            ws_buf = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)
            fr = W.rope_freqs_rows(f, a.m)
            run(lambda: NAT.check(NAT.LIB.w8a8_gemm_dequant_rms_rope(
                _vp(q), a.k, _vp(wq), a.k, _vp(xs), ctypes.byref(ep), _vp(y), a.n, a.m, a.n, a.k,
                rc, _vp(nw), 1 if rc != 128 else 0, _vp(fr), 1e-6, a.split_k,
                _vp(ws_buf) if nbytes else None, nbytes, ctypes.byref(c), _stream(dev))))
        elif a.kernel == "gemm_s32":
            q, _ = W.quantize_int8_rowwise(x)
            run(lambda: W.int8_gemm_s32(q, wq, config=cfg))
        elif a.kernel == "mxfp8_gemm":
            aq, asf = W.quantize_mxfp8(x)
            bq, bsf = W.quantize_mxfp8(w)
            run(lambda: W.mxfp8_linear(aq, asf, bq, bsf, b, out_dtype=torch.bfloat16, config=cfg))
        elif a.kernel == "gemv_q":
            # the GEMV alone, on activation codes quantised beforehand
            q, xs = W.quantize_int8_rowwise(x)
            run(lambda: W.int8_gemv(q, wq, xs, ws, b))
        elif a.kernel in ("gemm", "gemm_gelu", "gemv"):
            act = "gelu_tanh" if a.kernel == "gemm_gelu" else None
            if a.time and a.kernel != "gemv":
                # time the GEMM alone on pre-quantised activations
                import ctypes
                from imagine_b200 import _native as NAT
                from imagine_b200.linear import _config, _epilogue, _gemm_dequant, _stream, _vp
                q, xs = W.quantize_int8_rowwise(x)
                y = torch.empty((a.m, a.n), dtype=torch.bfloat16, device=dev)
                ep = _epilogue(ws, b, None, None, "eager", act, a.n, a.n)
                c = _config(cfg)
                if a.tiled:
                    tw = W.pack_weight_tiles(wq)
                    sk = None if a.split_k == 0 else a.split_k
                    run(lambda: _gemm_dequant(q, tw, xs.reshape(-1), ep, y, torch.bfloat16, a.m,
                                              a.n, a.k, c, sk, _stream(dev)))
                elif a.split_k != 1:
                    sk = None if a.split_k == 0 else a.split_k
                    run(lambda: _gemm_dequant(q, wq, xs.reshape(-1), ep, y, torch.bfloat16, a.m,
                                              a.n, a.k, c, sk, _stream(dev)))
                else:
                    run(lambda: NAT.check(NAT.LIB.w8a8_gemm_dequant(
                        _vp(q), a.k, _vp(wq), a.k, _vp(xs), ctypes.byref(ep), _vp(y), NAT.BF16, a.n,
                        a.m, a.n, a.k, ctypes.byref(c), _stream(dev))))
            else:
                run(lambda: W.int8_linear(x, wq, ws, b, output_act=act, config=cfg))
        else:
            sa = (x.abs().max().float() / 448).reshape(1)
            sw = (w.abs().max().float() / 448).reshape(1)
            aq = W.quantize_per_tensor_fp8(x, sa)
            wq8 = W.quantize_per_tensor_fp8(w, sw)
            run(lambda: W.fp8_linear(aq, sa, wq8, sw, b, config=cfg))
    torch.cuda.synchronize()
    err = W.device_error()
    if err:
        raise SystemExit(f"device error {err}")
    msg = (f"ok {a.kernel} {a.m} {a.k} {a.n} block_n={a.block_n} cta_group={a.cta_group} "
           f"split_k={a.split_k}" + (" tiled" if a.tiled else ""))
    if times:
        t = sorted(times)[len(times) // 2]
        ops = 2.0 * a.m * a.n * a.k
        msg += f" median_ms={t:.4f}"
        if a.kernel == "rms_rope":
            nbytes = 2 * 2 * a.m * a.k * 2 + a.m * 64 * 16
            msg += f" GB/s={nbytes / t / 1e6:.1f}"
        elif a.kernel in ("gemv", "gemv_q"):
            nbytes = a.n * a.k + 2 * (a.m * a.k + a.m * a.n) + 4 * a.n
            msg += f" GB/s={nbytes / t / 1e6:.1f}"
        elif a.kernel.startswith("sampler_"):
            # algorithmic bytes per element: Euler x in/out 8 + two bf16
            # outputs 4; ER-SDE stage 3 with noise adds history in/out 16 and noise 4
            per = 12 if a.kernel == "sampler_euler" else 32
            msg += f" GB/s={a.m * a.k * per / t / 1e6:.1f}"
        elif a.kernel == "dit_step":
            msg += f" blocks={a.blocks}"
        elif a.kernel not in ("quantize", "convrot", "rms_rope", "modulated"):
            msg += f" TOPS={ops / t / 1e9:.1f}"
        else:
            msg += f" GB/s={(a.m * a.k * 3 + 4 * a.m) / t / 1e6:.1f}"
    print(msg)


def _timed(fn, iters, flush, clean):
    """Median CUDA-event time (ms) of fn over iters calls, L2 flushed before
    each, after two warm-up calls."""
    fn()
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        torch.cuda._sleep(200000)
        flush.zero_()
        clean.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return sorted(times)[len(times) // 2]


def compare_libraries(a, dev, g, flush, clean):
    import json

    iters = max(a.iters, 5)
    if flush is None:
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        clean = torch.ones_like(flush)
    out = {"l2": "flushed before every call", "iters": iters, "stat": "median ms", "shapes": {}}
    for m, k, n in ((5600, 3072, 12288), (5600, 3072, 3072)):
        ops = 2.0 * m * n * k
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        row = {}

        def rec(name, fn):
            try:
                t = _timed(fn, iters, flush, clean)
                row[name] = {"ms": round(t, 4), "TOPS": round(ops / t / 1e9, 1)}
            except Exception as e:  # a library form this torch build does not offer
                row[name] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"}

        # INT8: int32 product, and the whole linear (dequant + bias to bf16)
        wq, ws = W.quantize_weight(w)
        q, xs = W.quantize_int8_rowwise(x)
        rec("int8_s32_ours", lambda: W.int8_gemm_s32(q, wq))
        wt = wq.t()
        rec("int8_s32_cublaslt_int_mm", lambda: torch._int_mm(q, wt))
        rec("int8_linear_ours_fused", lambda: W.int8_linear(x, wq, ws, b))

        def cublas_route():
            qq, sx = W.quantize_int8_rowwise(x)
            acc = torch._int_mm(qq, wt)
            return (acc.float() * (sx.reshape(-1, 1) * ws.reshape(1, -1))).to(torch.bfloat16) + b
        rec("int8_linear_cublaslt_then_aten_dequant", cublas_route)
        # FP8 per-tensor
        sa = (x.abs().max().float() / 448).reshape(1)
        sw = (w.abs().max().float() / 448).reshape(1)
        a8 = W.quantize_per_tensor_fp8(x, sa)
        w8 = W.quantize_per_tensor_fp8(w, sw)
        rec("fp8_tensorwise_ours", lambda: W.fp8_linear(a8, sa, w8, sw, b))
        sa0, sw0 = sa.reshape(()), sw.reshape(())
        rec("fp8_tensorwise_cublaslt_scaled_mm",
            lambda: torch._scaled_mm(a8, w8.t(), sa0, sw0, bias=b, out_dtype=torch.bfloat16))
        # MXFP8 (32-element blocks, e8m0 scales in the cuBLAS blocked layout)
        am, asf = W.quantize_mxfp8(x)
        wm, wsf = W.quantize_mxfp8(w)
        rec("mxfp8_ours", lambda: W.mxfp8_linear(am, asf, wm, wsf, b))
        e8 = getattr(torch, "float8_e8m0fnu", None)
        if e8 is not None:
            asf8, wsf8 = asf.view(e8), wsf.view(e8)
            rec("mxfp8_cublaslt_scaled_mm",
                lambda: torch._scaled_mm(am, wm.t(), asf8, wsf8, bias=b, out_dtype=torch.bfloat16))
        else:
            row["mxfp8_cublaslt_scaled_mm"] = {"unavailable": "no float8_e8m0fnu dtype"}
        out["shapes"][f"{m}x{k}x{n}"] = row
    err = W.device_error()
    if err:
        raise SystemExit(f"device error {err}")
    print(json.dumps(out))


if __name__ == "__main__":
    main()
