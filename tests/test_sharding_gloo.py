"""Multi-rank plumbing of the sharded step on CPU ranks (gloo): partition,
in-place all-gather of the NorMuon arena and of row-sharded tables, EMA
gather, and failure detection when a rank leaves. The per-rank compute is the
GPU engine (covered by the GPU tests); here each rank writes a known pattern
into the parameters it owns."""
import datetime
import os
import socket
import zlib

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sol_b200 import EmaWeights, build_optimizers, synth
from sol_b200.sharding import ShardedStep, assign_matrices, gram_cost

KW = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partition_is_balanced_and_deterministic(world):
    model = synth.SyntheticLM(synth.C2, device="meta")
    from sol_b200.routing import route_params
    mats = route_params(model.named_parameters())[0]
    shapes = [tuple(p.shape) for p in mats]
    owner, load = assign_matrices(shapes, world)
    assert owner == assign_matrices(shapes, world)[0]
    assert sorted(set(owner)) == list(range(world))
    total = sum(gram_cost(s) for s in shapes)
    biggest = max(gram_cost(s) for s in shapes)
    assert max(load) <= total / world + biggest  # LPT bound
    owner2, load2 = assign_matrices(shapes, world, "runs")
    assert owner2 == assign_matrices(shapes, world, "runs")[0]
    assert sorted(set(owner2)) == list(range(world))
    # shape runs: every rank holds at most three GEMM-path shapes (the 8 x 1024
    # gates run in their own one-CTA kernel)
    for r in range(world):
        assert len({shapes[i] for i in range(len(shapes)) if owner2[i] == r and min(shapes[i]) > 32}) <= 3


def _expected(name, shape, dtype):
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    return torch.randn(shape, generator=g).to(dtype)


def _worker(rank, world, port, mode, q, waves=1, assignment="lpt"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        model = synth.SyntheticLM(synth.MICRO, seed=0)
        muon, adamw = build_optimizers(model, **KW)
        ema = EmaWeights(model, 0.999)
        sharded = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, min_rows_shard=16, waves=waves,
                              assignment=assignment)
        named = list(model.named_parameters())
        # "step": each rank writes the final values of what it owns
        with torch.no_grad():
            for n, p in named:
                full = _expected(n, p.shape, p.dtype)
                if id(p) in sharded.owner:
                    if sharded.owner[id(p)] == rank:
                        p.copy_(full)
                    else:
                        p.zero_()
                elif any(p is t for t in sharded.row_sharded):
                    start, cnt = adamw._owned_slices[id(p)]
                    p.zero_()
                    p.view(-1)[start:start + cnt].copy_(full.view(-1)[start:start + cnt])
                else:
                    p.copy_(full)  # replicated: every rank computes it
        if mode == "leave" and rank == world - 1:
            q.put((rank, "left"))
            return  # leaves between steps, before the exchange
        try:
            sharded.gather()
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error: " + type(e).__name__))
            return
        bad = [n for n, p in named if not torch.equal(p.data, _expected(n, p.shape, p.dtype))]
        # EMA shadows: owners set a pattern, gather_ema completes the others
        with torch.no_grad():
            for i, (n, p) in enumerate(named):
                if i not in ema._skip:
                    ema.shadow[i].copy_(_expected(n, p.shape, torch.float32))
        sharded.gather_ema()
        bad_ema = [n for i, (n, p) in enumerate(named)
                   if not torch.equal(ema.shadow[i], _expected(n, p.shape, torch.float32))]
        q.put((rank, {"bad": bad, "bad_ema": bad_ema, "owned": len(muon._owned)}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, mode, waves=1, assignment="lpt"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q, waves, assignment)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=120)
        out[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,waves,assignment", [(2, 1, "lpt"), (3, 1, "lpt"), (2, 2, "runs"), (3, 3, "lpt")])
def test_gather_reassembles_every_parameter(world, waves, assignment):
    """Wave-major arena (waves > 1) and shape-run assignment included."""
    out = _run(world, "ok", waves, assignment)
    assert sorted(out) == list(range(world))
    for r, v in out.items():
        assert v["bad"] == [], (r, v["bad"])
        assert v["bad_ema"] == [], (r, v["bad_ema"])
    assert sum(v["owned"] for v in out.values()) == 3 * 5  # MICRO: 3 layers x 5 NorMuon matrices


def test_rank_leaving_is_detected_not_hung():
    """A rank that leaves before the exchange makes the others' gather fail
    within the process-group timeout instead of hanging."""
    out = _run(2, "leave")
    assert out[1] == "left"
    assert isinstance(out[0], str) and out[0].startswith("error"), out[0]


def _reduce_worker(rank, world, port, average, q, waves=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        model = synth.SyntheticLM(synth.MICRO, seed=0)
        muon, adamw = build_optimizers(model, **KW)
        ema = EmaWeights(model, 0.999)
        sharded = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, min_rows_shard=16, waves=waves)
        named = list(model.named_parameters())
        with torch.no_grad():
            for n, p in named:
                p.grad = _expected(n + f"#{rank}", p.shape, p.dtype)
        sharded.reduce_gradients(average=average)
        worst = 0.0
        checked = 0
        for n, p in named:
            exact = sum(_expected(n + f"#{r}", p.shape, p.dtype).float() for r in range(world))
            if average:
                exact = exact / world
            want = exact.to(p.dtype).float()
            got = p.grad.float()
            if id(p) in sharded.owner:
                if sharded.owner[id(p)] != rank:
                    continue
            elif any(p is t for t in sharded.row_sharded):
                start, cnt = adamw._owned_slices[id(p)]
                want = want.view(-1)[start:start + cnt]
                got = got.view(-1)[start:start + cnt]
            # at most one bf16 rounding step apart (fp32 sums in another order)
            ulp = torch.clamp(want.abs(), min=1e-30) * 2.0 ** -7
            worst = max(worst, float(((got - want).abs() / ulp).max()))
            checked += 1
        q.put((rank, {"worst_ulps": worst, "checked": checked}))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world,average,waves", [(2, False, 1), (2, True, 1), (3, True, 1), (3, True, 2)])
def test_reduce_gradients_sums_what_each_rank_reads(world, average, waves):
    """Each rank holds its own gradients; after reduce_gradients every rank
    holds the sum (or mean) over ranks of the gradients its step reads."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, average, q, waves)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=180)
            out[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert isinstance(out[r], dict), out[r]
        assert out[r]["checked"] > 0
        limit = 0.0 if world == 2 else 1.0  # two addends: one rounding, bit-exact
        assert out[r]["worst_ulps"] <= limit, out[r]


@pytest.mark.parametrize("world,waves,assignment", [(2, 1, "lpt"), (3, 1, "lpt"), (4, 1, "lpt"), (8, 1, "lpt"),
                                                    (2, 2, "runs"), (4, 2, "runs"), (8, 3, "lpt")])
def test_owned_regions_are_disjoint_and_cover_every_update(world, waves, assignment):
    """The regions each rank pushes (sharded step) tile every NorMuon matrix and
    every row-sharded table exactly once; each wave's owned set is exactly the
    rank's matrices in that wave's arena region."""
    steps = []
    for rank in range(world):
        model = synth.SyntheticLM(synth.MICRO, seed=0)
        muon, adamw = build_optimizers(model, **KW)
        steps.append(ShardedStep(model, muon, adamw, None, world=world, rank=rank, min_rows_shard=16,
                                 exchange="nccl", waves=waves, assignment=assignment))
    ref = steps[0]
    bufs = ref.buffers()
    covered = [torch.zeros(b.numel() * b.element_size(), dtype=torch.int32) for b in bufs]
    for st in steps:
        assert [b.numel() for b in st.buffers()] == [b.numel() for b in bufs]
        for k, off, nbytes in st.owned_regions(st.rank):
            covered[k][off:off + nbytes] += 1
    assert all(int(c.max()) <= 1 for c in covered)  # disjoint
    # every byte of every NorMuon matrix and every table is pushed by one rank
    base = ref.arena.data_ptr()
    es = ref.arena.element_size()
    for p in (p for g in ref.muon.param_groups for p in g["params"]):
        off = p.data.data_ptr() - base
        assert int(covered[0][off:off + p.numel() * es].min()) == 1
    for k in range(1, len(bufs)):
        assert int(covered[k].min()) == 1
    for st in steps:
        assert set().union(*st.wave_owned) == st.owned_all
        assert sum(len(w) for w in st.wave_owned) == len(st.owned_all)
        mparams = {id(p): p for g in st.muon.param_groups for p in g["params"]}
        b0, es0 = st.arena.data_ptr(), st.arena.element_size()
        for w, ids in enumerate(st.wave_owned):
            wbase, chunk, _ = st.arena_waves[w]
            lo = (wbase + st.rank * chunk) * es0
            for i in ids:
                off = mparams[i].data.data_ptr() - b0
                assert lo <= off and off + mparams[i].numel() * es0 <= lo + chunk * es0
