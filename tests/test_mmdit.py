"""The MMDiT harness (imagine_b200.mmdit) on the CPU oracle: positions,
timestep embedding, placement, and the multi-rank forms (CFG branches on
separate ranks, tensor parallelism inside a branch) against the one-rank
model, as gloo ranks."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from imagine_b200 import mmdit as M

TINY = M.MMDiTConfig(hidden=256, heads=2, head_dim=128, mlp_hidden=512, blocks=2,
                     context_dim=256, time_dim=64)


def test_sequence_ids_follow_assemble_sequence():
    txt, img = M.sequence_ids(4, 3, 4)
    assert txt.tolist() == [[i, i, i] for i in range(4)]
    # frame index = text length; rows centred (h - h//2 subtracted), columns likewise
    assert img.shape == (12, 3)
    assert img[:, 0].unique().tolist() == [4.0]
    assert img[:, 1].reshape(3, 4)[:, 0].tolist() == [-2.0, -1.0, 0.0]
    assert img[:, 2].reshape(3, 4)[0].tolist() == [-2.0, -1.0, 0.0, 1.0]


def test_rope_freqs_are_rotations_of_pos_times_omega():
    ids = torch.tensor([[3.0, -2.0, 5.0], [0.0, 1.0, -7.0]])
    f = M.rope_freqs(ids, (16, 56, 56))
    assert f.shape == (2, 64, 2, 2) and f.dtype == torch.float32
    # pair j of axis 1 (offset 8 pairs): angle = pos * theta^(-2j/56)
    j = 5
    ang = -2.0 * 10000.0 ** (-(2 * j) / 56)
    want = torch.tensor([[math.cos(ang), -math.sin(ang)], [math.sin(ang), math.cos(ang)]])
    assert torch.allclose(f[0, 8 + j], want, atol=1e-6)
    # every block is a rotation
    det = f[..., 0, 0] * f[..., 1, 1] - f[..., 0, 1] * f[..., 1, 0]
    assert torch.allclose(det, torch.ones_like(det), atol=1e-6)


def test_timestep_embedding_matches_formula():
    t = torch.tensor([0.25, 0.9])
    e = M.timestep_embedding(t, 8)
    freq = torch.exp(torch.arange(4, dtype=torch.float32) * -math.log(10000.0) / 4)
    args = t[:, None] * 1000 * freq[None]
    assert torch.allclose(e, torch.cat([args.cos(), args.sin()], -1))


def test_patchify_roundtrip():
    x = torch.randn(2, 16, 8, 12)
    p = M.patchify(x, 2)
    assert p.shape == (2, 24, 64)
    assert torch.equal(p[0, 0, :4], x[0, 0, :2, :2].reshape(-1))
    assert torch.equal(M.unpatchify(p, 2, 16, 8, 12), x)


@pytest.mark.parametrize("world,expect", [
    (1, [(1, 0, 0)]),
    (2, [(1, 0, 0), (1, 1, 0)]),
    (4, [(2, 0, 0), (2, 0, 1), (2, 1, 0), (2, 1, 1)]),
    (8, [(4, 0, 0), (4, 0, 1), (4, 0, 2), (4, 0, 3), (4, 1, 0), (4, 1, 1), (4, 1, 2), (4, 1, 3)]),
])
def test_placement(world, expect):
    got = [(p.tp, p.branch, p.tp_rank) for p in (M.placement(world, r) for r in range(world))]
    assert got == expect
    with pytest.raises(ValueError):
        M.placement(3, 0)
    assert M.placement(4, 1).sequence_parallel and not M.placement(4, 1).tensor_parallel
    assert M.placement(4, 1, "tensor").tensor_parallel
    assert not M.placement(2, 1).sequence_parallel and not M.placement(2, 1, "tensor").tensor_parallel


def _oracle_model(tp_rank=0, tp_world=1, group=None, cfg=TINY, seed=0):
    from tests._mmdit_oracle import OracleOps

    ops = OracleOps()
    params = M.random_params(cfg, ops, "cpu", seed=seed, tp_rank=tp_rank, tp_world=tp_world)
    return M.MMDiT(params, ops, group)


def _inputs(cfg=TINY, b=1, h=8, w=8, st=8, seed=5):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(b, cfg.latent_channels, h, w, generator=g).to(torch.bfloat16)
    ctx_c = torch.randn(b, st, cfg.context_dim, generator=g).to(torch.bfloat16)
    ctx_u = torch.randn(b, st, cfg.context_dim, generator=g).to(torch.bfloat16)
    return lat, ctx_c, ctx_u


def test_oracle_forward_shapes_and_weight_shards():
    model = _oracle_model()
    lat, ctx, _ = _inputs(b=2)
    out = model.forward(lat, torch.tensor([0.7, 0.7]), ctx)
    assert out.shape == lat.shape and out.dtype == torch.bfloat16
    assert torch.isfinite(out.float()).all()
    full = M.random_params(TINY, model.ops, "cpu", seed=0)
    half = M.random_params(TINY, model.ops, "cpu", seed=0, tp_rank=1, tp_world=2)
    b0, h0 = full.blocks[0].img, half.blocks[0].img
    c = TINY.hidden
    assert torch.equal(h0.qkv.w[: c // 2], b0.qkv.w[c // 2: c])          # q rows of head 1
    assert torch.equal(h0.qkv.w[c // 2: c], b0.qkv.w[c + c // 2: 2 * c])  # k rows of head 1
    assert torch.equal(h0.out.w, b0.out.w[:, c // 2:])
    assert torch.equal(h0.down.w, b0.down.w[:, TINY.mlp_hidden // 2:])
    assert torch.equal(half.mod_img.w, full.mod_img.w[full.mod_img.w.shape[0] // 2:])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, mode):
    from tests._mmdit_oracle import OracleOps

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pl = M.placement(world, rank, mode)
        groups = M.ProcessGroups(pl)
        model = M.build_model(TINY, OracleOps(), "cpu", pl, groups, seed=0)
        lat, ctx_c, ctx_u = _inputs()
        fn = M.cfg_model(model, pl, groups, ctx_c, ctx_u)
        oc, ou = fn(lat.float(), torch.tensor([0.55]), True)
        q.put((rank, oc, ou))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, "sequence"), (4, "sequence"), (4, "tensor"),
                                        (8, "sequence")])
def test_multi_rank_step_equals_one_rank(world, mode):
    """CFG branches on separate ranks (world 2) and, on world 4, each branch
    split over 2 ranks by image tokens (sequence) or by heads and MLP columns
    (tensor), and on world 8 the image tokens split 4 ways, give the one-rank
    batched model's predictions bit for bit."""
    model = _oracle_model()
    lat, ctx_c, ctx_u = _inputs()
    pl = M.placement(1, 0)
    want_c, want_u = M.cfg_model(model, pl, M.ProcessGroups(pl), ctx_c, ctx_u)(
        lat.float(), torch.tensor([0.55]), True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, oc, ou in got:
        assert torch.equal(oc.view(torch.int16), want_c.view(torch.int16)), rank
        assert torch.equal(ou.view(torch.int16), want_u.view(torch.int16)), rank
