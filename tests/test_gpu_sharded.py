"""Sharded step on two GPUs (NCCL process group, copy-engine peer pushes):
every rank's parameters and, after gather_ema(), its EMA shadows must be
bit-identical to the unsharded engine run on the same seeded inputs, since
placement never changes a matrix's arithmetic. Needs two GPUs; skipped on a
one-GPU box. The ranks run as spawned child processes with a short
process-group timeout, so a rank that fails ends the others' collectives
with an error instead of a wait."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

KW = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)
STEPS = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, exchange, q, dp=False, waves=1, assignment="lpt", between=False):
    import torch.distributed as dist

    from sol_b200 import EmaWeights, build_optimizers, synth
    from sol_b200.sharding import ShardedStep
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sharded = None
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        cfg = synth.MICRO
        model = synth.SyntheticLM(cfg, device=dev, seed=0)
        muon, adamw = build_optimizers(model, adam_master="bf16_mt", **KW)
        ema = EmaWeights(model, 0.999)
        sharded = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, min_rows_shard=16,
                              exchange=exchange, waves=waves, assignment=assignment, adamw_between_waves=between)
        ref = synth.SyntheticLM(cfg, device=dev, seed=0)
        rmuon, radamw = build_optimizers(ref, adam_master="bf16_mt", **KW)
        rema = EmaWeights(ref, 0.999)
        for step in range(STEPS):
            if dp:
                # data parallel: each rank its own gradients; the reference
                # steps on their mean (an fp32 sum of two bf16 values is exact,
                # the halving too: one rounding, as in reduce_gradients)
                mine = synth.make_grads(model, step, seed=rank)
                both = [synth.make_grads(model, step, seed=r) for r in range(world)]
                grads = [(sum(g[i].float() for g in both) / world).to(mine[i].dtype) for i in range(len(mine))]
                synth.set_grads(model, [g.clone() for g in mine])
                synth.set_grads(ref, grads)
                sharded.reduce_gradients(average=True)
            else:
                grads = synth.make_grads(model, step, seed=0)
                synth.set_grads(model, [g.clone() for g in grads])
                synth.set_grads(ref, grads)
            sharded.step()
            rmuon.step()
            radamw.step()
            rema.update()
        torch.cuda.synchronize()
        named, rnamed = list(model.named_parameters()), list(ref.named_parameters())
        bad = [n for (n, p), (_, r) in zip(named, rnamed) if not torch.equal(p.data, r.data)]
        sharded.gather_ema()
        torch.cuda.synchronize()
        bad_ema = [n for (n, _), s, r in zip(named, ema.shadow, rema.shadow) if not torch.equal(s, r)]
        # checkpoint path: every rank's optimizer state completed from the owners
        sharded.gather_state()
        torch.cuda.synchronize()
        bad_state = []
        for a, b in ((muon, rmuon), (adamw, radamw)):
            pa = [p for g in a.param_groups for p in g["params"]]
            pb = [p for g in b.param_groups for p in g["params"]]
            for i, (p, r) in enumerate(zip(pa, pb)):
                for k, v in b.state[r].items():
                    if k != "step" and not torch.equal(a.state[p][k], v):
                        bad_state.append((type(a).__name__, i, k))
        q.put((rank, {"exchange": sharded.exchange, "bad": bad, "bad_ema": bad_ema, "bad_state": bad_state,
                      "owned": len(muon._owned)}))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        if sharded is not None and dist.is_initialized():
            try:
                sharded.close()
            except Exception:  # noqa: BLE001
                pass
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("exchange,dp,waves,assignment,between", [
    ("ce", False, 1, "lpt", False), ("hybrid", False, 1, "lpt", False), ("nccl", False, 1, "lpt", False),
    ("auto", True, 1, "lpt", False), ("ce", False, 2, "runs", False), ("hybrid", False, 2, "lpt", False),
    ("nccl", True, 2, "runs", False), ("hybrid", False, 2, "lpt", True), ("ce", False, 2, "lpt", True)])
def test_sharded_step_bit_identical_to_single_gpu(exchange, dp, waves, assignment, between):
    """dp: each rank steps on its own gradients after reduce_gradients; the
    single-GPU reference steps on their mean. waves > 1: each wave's weights
    are exchanged while the next wave computes."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q, dp, waves, assignment, between))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=300)
            out[r] = v
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        v = out[r]
        assert isinstance(v, dict), (r, v)
        assert v["exchange"] == (exchange if exchange != "auto" else "ce")
        assert v["bad"] == [], (r, v["bad"])
        assert v["bad_ema"] == [], (r, v["bad_ema"])
        assert v["bad_state"] == [], (r, v["bad_state"])
    assert sum(v["owned"] for v in out.values()) == 3 * 5  # MICRO: 3 layers x 5 NorMuon matrices
