"""Checkpoints in the reference's layout (transformer_lm/modules.py:538-560;
ema_final.pt at train_sol.py:542-549): file layout and state dtypes on the
CPU, gather of a sharded rank's state on gloo ranks, and on the GPU a resumed
run that is bit-identical to an uninterrupted one."""
import datetime
import io
import os
import socket
import zlib

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sol_b200 import EmaWeights, build_optimizers, synth
from sol_b200.checkpoint import load_checkpoint, load_ema, save_checkpoint, save_ema
from sol_b200.sharding import ShardedStep

KW = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)


def _pattern(name, shape, dtype, salt=0):
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()) + salt)
    return torch.randn(shape, generator=g).to(dtype)


def _fill_state(model, muon, adamw, owned=None, rows=None):
    """Writes name-derived patterns into the optimizer state (all of it, or the
    matrices in `owned` and the `rows` slices of the tables)."""
    names = {id(p): n for n, p in model.named_parameters()}
    for g in muon.param_groups:
        for p in g["params"]:
            if owned is not None and id(p) not in owned:
                continue
            st = muon._init_state(p)
            for k in st:
                st[k].copy_(_pattern(names[id(p)] + k, st[k].shape, st[k].dtype))
    for g in adamw.param_groups:
        for p in g["params"]:
            st = adamw._init_state(p)
            for k in ("exp_avg", "exp_avg_sq", "mant_rem"):
                if k not in st:
                    continue
                full = _pattern(names[id(p)] + k, st[k].shape, st[k].dtype)
                if rows is not None and id(p) in rows:
                    start, cnt = rows[id(p)]
                    st[k].view(-1)[start:start + cnt].copy_(full.view(-1)[start:start + cnt])
                else:
                    st[k].copy_(full)
            st["step"].fill_(7.0)
            adamw._steps[id(p)] = 7


def test_checkpoint_layout_and_dtypes_round_trip():
    model = synth.SyntheticLM(synth.MICRO, seed=0)
    muon, adamw = build_optimizers(model, adam_master="bf16_mt", **KW)
    ema = EmaWeights(model, 0.999)
    _fill_state(model, muon, adamw)
    for i, s in enumerate(ema.shadow):
        s.copy_(_pattern(f"ema{i}", s.shape, torch.float32))
    buf, ebuf = io.BytesIO(), io.BytesIO()
    save_checkpoint(model, muon, 123, buf, adamw=adamw)
    save_ema(model, ema, ebuf)
    buf.seek(0)
    ebuf.seek(0)
    obj = torch.load(io.BytesIO(buf.getvalue()), weights_only=False)
    assert set(obj) == {"model", "optimizer", "iteration", "adamw"}
    assert set(obj["optimizer"]) == {"state", "param_groups"}
    # NorMuon state keeps the reference's names and the fp32 v_row of bf16 matrices
    st0 = obj["optimizer"]["state"][0]
    assert set(st0) == {"momentum_buffer", "v_row", "mant_rem"}
    assert st0["v_row"].dtype == torch.float32 and st0["momentum_buffer"].dtype == torch.bfloat16

    # a plain torch optimizer with the same groups (what the reference's loader
    # hands the file to) accepts the NorMuon state
    class Plain(torch.optim.Optimizer):
        def __init__(self, params):
            super().__init__(params, {})
    model2 = synth.SyntheticLM(synth.MICRO, seed=1)
    plain = Plain([{"params": [p for g in build_optimizers(model2, **KW)[0].param_groups for p in g["params"]]}])
    plain.load_state_dict({"state": obj["optimizer"]["state"],
                           "param_groups": [dict(obj["optimizer"]["param_groups"][0], params=list(
                               range(len(obj["optimizer"]["param_groups"][0]["params"]))))]})

    model3 = synth.SyntheticLM(synth.MICRO, seed=2)
    muon3, adamw3 = build_optimizers(model3, adam_master="bf16_mt", **KW)
    ema3 = EmaWeights(model3, 0.999)
    assert load_checkpoint(buf, model3, muon3, adamw=adamw3) == 123
    load_ema(ebuf, model3, ema3)
    for (n, p), (_, q) in zip(model.named_parameters(), model3.named_parameters()):
        assert torch.equal(p, q), n
    for a, b in ((muon, muon3), (adamw, adamw3)):
        pa = [p for g in a.param_groups for p in g["params"]]
        pb = [p for g in b.param_groups for p in g["params"]]
        for p, q in zip(pa, pb):
            for k, v in a.state[p].items():
                w = b.state[q][k]
                assert w.dtype == v.dtype and torch.equal(w, v), k
    assert all(adamw3._steps[id(p)] == 7 for g in adamw3.param_groups for p in g["params"])
    for s, t in zip(ema.shadow, ema3.shadow):
        assert torch.equal(s, t)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        model = synth.SyntheticLM(synth.MICRO, seed=0)
        muon, adamw = build_optimizers(model, adam_master="bf16_mt", **KW)
        ema = EmaWeights(model, 0.999)
        sharded = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, min_rows_shard=16)
        rows = {id(p): adamw._owned_slices[id(p)] for p in sharded.row_sharded}
        _fill_state(model, muon, adamw, owned=muon._owned, rows=rows)
        sharded.gather_state()
        ref = synth.SyntheticLM(synth.MICRO, seed=0)
        rmuon, radamw = build_optimizers(ref, adam_master="bf16_mt", **KW)
        _fill_state(ref, rmuon, radamw)
        bad = []
        for a, b in ((muon, rmuon), (adamw, radamw)):
            pa = [p for g in a.param_groups for p in g["params"]]
            pb = [p for g in b.param_groups for p in g["params"]]
            for i, (p, r) in enumerate(zip(pa, pb)):
                for k, v in b.state[r].items():
                    if k != "step" and not torch.equal(a.state[p][k], v):
                        bad.append((type(a).__name__, i, k))
        sharded.drop_unowned_state()
        left = len(muon.state)
        q.put((rank, {"bad": bad, "left": left, "owned": len(muon._owned)}))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_gather_state_completes_every_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
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
        assert out[r]["bad"] == [], out[r]["bad"]
        assert out[r]["left"] == out[r]["owned"]


@pytest.mark.gpu
def test_resume_is_bit_identical(cuda):
    """5 uninterrupted steps == 3 steps, checkpoint, fresh engine, load, 2 steps."""
    def engine():
        model = synth.SyntheticLM(synth.MICRO, device=cuda, seed=0)
        muon, adamw = build_optimizers(model, adam_master="bf16_mt", **KW)
        return model, muon, adamw, EmaWeights(model, 0.999)

    def run(eng, steps):
        model, muon, adamw, ema = eng
        for k in steps:
            synth.set_grads(model, synth.make_grads(model, k, seed=0))
            muon.step()
            adamw.step()
            ema.update()

    a = engine()
    run(a, range(5))
    b = engine()
    run(b, range(3))
    buf, ebuf = io.BytesIO(), io.BytesIO()
    save_checkpoint(b[0], b[1], 3, buf, adamw=b[2])
    save_ema(b[0], b[3], ebuf)
    buf.seek(0)
    ebuf.seek(0)
    c = engine()
    assert load_checkpoint(buf, c[0], c[1], adamw=c[2]) == 3
    load_ema(ebuf, c[0], c[3])
    run(c, range(3, 5))
    torch.cuda.synchronize()
    for (n, p), (_, q) in zip(a[0].named_parameters(), c[0].named_parameters()):
        assert torch.equal(p, q), n
    for x, y in ((a[1], c[1]), (a[2], c[2])):
        px = [p for g in x.param_groups for p in g["params"]]
        py = [p for g in y.param_groups for p in g["params"]]
        for p, q in zip(px, py):
            for k, v in x.state[p].items():
                assert torch.equal(v, y.state[q][k]), (type(x).__name__, k)
    for s, t in zip(a[3].shadow, c[3].shadow):
        assert torch.equal(s, t)
