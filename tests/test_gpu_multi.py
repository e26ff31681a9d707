"""Tensor-parallel linears on 2, 4 and 8 GPUs with the native kernels: the NCCL
forms (column- and row-parallel) and the column-parallel linear whose
all-gather is fused into the GEMM epilogue (chunk copies over NVLink) and the
row-parallel linear whose reduce-scatter is fused into the GEMM epilogue must
all equal the single-GPU int8_linear bit for bit -- including the AdaLN
modulation linear (2 rows of SiLU(temb), 3072 -> 18432) column-parallel
through the fused path; on 2 GPUs CFG-parallel sampling (one branch per GPU)
must give the single-GPU latent.  Each size skips on boxes with fewer GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import imagine_b200 as W
        from imagine_b200 import tensor_parallel as TP

        g = torch.Generator().manual_seed(3)
        m, k, n = 600, 3072, 1536
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        wq, ws = W.quantize_weight(w)
        ref = W.int8_linear(x, wq, ws, b)
        col = TP.ColumnParallelInt8Linear(wq, ws, b)
        row = TP.RowParallelInt8Linear(wq, ws, b)
        y_col = col(x)
        y_row = row(row.shard_input(x))
        # the all-gather fused into the GEMM (peer stores over NVLink): two
        # calls with different inputs (epochs 1 and 2), and the GELU epilogue
        fused = TP.ColumnParallelInt8Linear(wq, ws, b, fused=True)
        fused_gelu = TP.ColumnParallelInt8Linear(wq, ws, b, fused=True, output_act="gelu_tanh")
        assert fused.fused and fused_gelu.fused
        x2 = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        ok_fused = True
        for xi in (x, x2, x):
            want = W.int8_linear(xi, wq, ws, b)
            ok_fused &= torch.equal(fused(xi).view(torch.int16), want.view(torch.int16))
            want = W.int8_linear(xi, wq, ws, b, output_act="gelu_tanh")
            ok_fused &= torch.equal(fused_gelu(xi).view(torch.int16), want.view(torch.int16))
        torch.cuda.synchronize()
        ok_fused &= W.device_error() == 0
        # the all-reduce fused into the row-parallel GEMM (int32 partial chunks
        # sent to their rows' owners, summed there, rows handed back): three
        # calls, bf16 and fp32 outputs
        rowf = TP.RowParallelInt8Linear(wq, ws, b, fused=True)
        assert rowf.fused
        for xi in (x, x2, x):
            want = W.int8_linear(xi, wq, ws, b)
            ok_fused &= torch.equal(rowf(rowf.shard_input(xi)).view(torch.int16),
                                    want.view(torch.int16))
        want32 = W.int8_linear(x2, wq, ws, b.float(), out_dtype=torch.float32)
        ok_fused &= torch.equal(rowf(rowf.shard_input(x2), out_dtype=torch.float32), want32)
        torch.cuda.synchronize()
        ok_fused &= W.device_error() == 0
        # the AdaLN modulation linear: 2 rows (CFG) of SiLU(temb), 3072 -> 18432,
        # column-parallel with the all-gather fused into the GEMM
        wm = (torch.randn(18432, k, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        bm = (torch.randn(18432, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        wmq, wms = W.quantize_weight(wm)
        s_temb = torch.nn.functional.silu(torch.randn(2, k, generator=g).to(torch.bfloat16)).to(dev)
        modf = TP.ColumnParallelInt8Linear(wmq, wms, bm, fused=True)
        assert modf.fused
        want = W.int8_linear(s_temb, wmq, wms, bm)
        for _ in range(2):
            ok_fused &= torch.equal(modf(s_temb).view(torch.int16), want.view(torch.int16))
        torch.cuda.synchronize()
        ok_fused &= W.device_error() == 0
        if world != 2:
            q.put((rank, torch.equal(y_col.view(torch.int16), ref.view(torch.int16)),
                   torch.equal(y_row.view(torch.int16), ref.view(torch.int16)), bool(ok_fused)))
            return
        # CFG-parallel sampling: rank r evaluates branch r, one all-gather of
        # the outputs, then the fused ER-SDE step on every rank -- the same
        # latent as both branches on one GPU
        from imagine_b200 import sampler as SM

        def branch(xx, ts, bb):
            t = ts.reshape(-1, 1, 1, 1)
            return (xx.mul(0.61).add(t.mul(0.5)) if bb == 0 else xx.mul(-0.23).sub(t)).to(
                torch.bfloat16)

        def noises():
            gg = torch.Generator().manual_seed(9)
            return lambda xx: torch.randn(xx.shape, generator=gg).to(dev)

        x0 = torch.randn(2, 16, 28, 50, generator=torch.Generator().manual_seed(5))
        sig = SM.FluxSampling().simple(6)
        y_par = SM.sample_er_sde(x0.to(dev), sig, SM.FluxSampling(), SM.cfg_parallel_model(branch),
                                 3.0, noise_like=noises())
        y_one = SM.sample_er_sde(x0.to(dev), sig, SM.FluxSampling(),
                                 lambda xx, ts, wu: (branch(xx, ts, 0), branch(xx, ts, 1)), 3.0,
                                 noise_like=noises())
        ok_fused &= torch.equal(y_par, y_one)
        q.put((rank, torch.equal(y_col.view(torch.int16), ref.view(torch.int16)),
               torch.equal(y_row.view(torch.int16), ref.view(torch.int16)), bool(ok_fused)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_nccl_bit_exact(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, col_ok, row_ok, fused_ok in results:
        assert col_ok and row_ok and fused_ok, (rank, col_ok, row_ok, fused_ok)
