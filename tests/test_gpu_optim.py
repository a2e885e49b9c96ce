"""Parity of the engine's optimizer step with the oracle (the reference's own
step restated on the CPU, pinned by tests/golden) and with torch's fused AdamW.

Tolerances (stated where they are checked):
  * AdamW / EMA element math: fp32 values within 2 ulp; bf16 values equal or
    one bf16 ulp apart where the fp32 result sits on a rounding boundary.
  * bf16 mantissa split / recombine: bit-exact given the same fp32 weight.
  * Orthogonalised NorMuon updates: relative Frobenius error of the cumulative
    update after 10 steps <= 1e-2 for fp32 parameters. The reference's
    orthogonaliser is bf16 Newton-Schulz; changing only the order of fp32
    accumulation inside its GEMMs moves its output by ~0.5-1.3 % (measured on
    the CPU by tests/test_host_cpu.py::test_bf16_newton_schulz_noise_floor), so
    for bf16 parameters the bound is 1.5e-2 with mantissa tracking and 2.5e-2
    without it (there every step also rounds the weight itself to bf16).
"""
import math

import pytest
import torch

from oracle import gram_ns_ref, ref_step
from sol_b200 import AdamW, EmaWeights, NorMuonGNS, _lib, build_optimizers, polar_express, synth

pytestmark = pytest.mark.gpu


def _ulp_f32(x):
    return torch.finfo(torch.float32).eps * x.abs().clamp_min(torch.finfo(torch.float32).tiny)


def assert_f32_ulps(a, b, ulps=2, what=""):
    a, b = a.float().cpu(), b.float().cpu()
    bad = (a - b).abs() > ulps * _ulp_f32(b) * 1.0001
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond {ulps} ulp; max |d| {(a - b).abs().max()}"


def assert_bf16_close(a, b, what="", min_exact=0.999):
    a, b = a.to(torch.bfloat16).cpu(), b.to(torch.bfloat16).cpu()
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    d = (ai - bi).abs()
    assert d.max() <= 1, f"{what}: bf16 values more than one ulp apart"
    assert (d == 0).float().mean() >= min_exact, f"{what}: too many 1-ulp differences"


def rel_fro(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return (torch.linalg.norm(a - b) / torch.linalg.norm(b).clamp_min(1e-30)).item()


# ------------------------------------------------------------------ AdamW ---
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_adamw_matches_torch_fused_cuda(cuda, dtype):
    """Reference mode == torch.optim.AdamW(fused=True) on the same device."""
    g = torch.Generator(device=cuda).manual_seed(0)
    shapes = [(333, 77), (1024,), (5, 64, 32), (), (7,), (4096, 64)]
    base = [torch.randn(s, generator=g, device=cuda) * 0.02 for s in shapes]
    p1 = [torch.nn.Parameter(b.clone().to(dtype)) for b in base]
    p2 = [torch.nn.Parameter(b.clone().to(dtype)) for b in base]
    groups = lambda ps: [{"params": ps[:3], "lr": 2.4e-2, "weight_decay": 0.0},  # noqa: E731
                         {"params": ps[3:5], "lr": 1e-2, "betas": (0.75, 0.95), "weight_decay": 0.1},
                         {"params": ps[5:], "lr": 3e-3}]
    ours = AdamW(groups(p1), betas=(0.9, 0.95), eps=1e-8, fused=True)
    ref = torch.optim.AdamW(groups(p2), betas=(0.9, 0.95), eps=1e-8, fused=True)
    for step in range(5):
        for a, b in zip(p1, p2):
            gr = (torch.randn(a.shape, generator=g, device=cuda) * 1e-3).to(dtype)
            a.grad, b.grad = gr.clone(), gr.clone()
        ours.step()
        ref.step()
    torch.cuda.synchronize()
    for a, b in zip(p1, p2):
        sa, sb = ours.state[a], ref.state[b]
        if dtype == torch.float32:
            assert_f32_ulps(a.data, b.data, what="param")
            assert_f32_ulps(sa["exp_avg"], sb["exp_avg"], what="exp_avg")
            assert_f32_ulps(sa["exp_avg_sq"], sb["exp_avg_sq"], what="exp_avg_sq")
        else:
            assert_bf16_close(a.data, b.data, "param")
            assert_bf16_close(sa["exp_avg"], sb["exp_avg"], "exp_avg")
            assert_bf16_close(sa["exp_avg_sq"], sb["exp_avg_sq"], "exp_avg_sq")
    sd = ours.state_dict()
    assert float(sd["state"][0]["step"]) == 5.0


def test_adamw_master_mode_vs_oracle(cuda):
    """bf16 params + bf16 remainder + fp32 moments + cautious decay vs the CPU
    restatement, one step at a time from identical state (6 steps: the oracle's
    state is copied into the engine before each step)."""
    g = torch.Generator().manual_seed(1)
    shapes = [(512, 96), (1000,), (3, 40, 24)]
    init = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    pg = [torch.nn.Parameter(x.to(torch.bfloat16).cuda()) for x in init]
    pc = [torch.nn.Parameter(x.to(torch.bfloat16)) for x in init]
    ours = AdamW(pg, lr=2.4e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, master="bf16_mt",
                 cautious_wd=True)
    orc = ref_step.MasterAdamW(pc, lr=2.4e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, cautious=True)
    for step in range(6):
        for a, b in zip(pg, pc):
            gr = (torch.randn(b.shape, generator=g) * 1e-3)
            gr[..., :3] *= 10
            gr = gr.to(torch.bfloat16)
            a.grad, b.grad = gr.cuda(), gr.clone()
        if step > 0:  # identical starting state
            for a, b, st in zip(pg, pc, orc.state):
                so = ours.state[a]
                a.data.copy_(b.data)
                so["mant_rem"].copy_(st["rem"])
                so["exp_avg"].copy_(st["m"])
                so["exp_avg_sq"].copy_(st["v"])
        w_before = [b.data.float() + (st["rem"].float() if st["rem"] is not None else 0) for b, st in zip(pc, orc.state)]
        ours.step()
        orc.step()
        torch.cuda.synchronize()
        for a, b, st, wb in zip(pg, pc, orc.state, w_before):
            so = ours.state[a]
            assert_f32_ulps(so["exp_avg"], st["m"], what="exp_avg")
            assert_f32_ulps(so["exp_avg_sq"], st["v"], what="exp_avg_sq")
            w_ours = a.data.float().cpu() + so["mant_rem"].float().cpu()
            w_orc = b.data.float() + st["rem"].float()
            # bf16 parameter + bf16 remainder resolves w to about 2^-16 |w|; the
            # bias corrections use powf on the GPU and torch.pow on the CPU (an ulp
            # apart at most), which moves the update by a few 1e-7 of itself, and
            # such a difference can move the remainder's bf16 rounding by one step.
            tol = 2.0 ** -15 * w_orc.abs() + 5e-7 * (w_orc - wb).abs() + 4 * _ulp_f32(w_orc)
            assert ((w_ours - w_orc).abs() <= tol).all(), f"reconstructed weight, step {step}"
            assert_bf16_close(a.data, b.data, "bf16 parameter", min_exact=0.999)


def test_mantissa_split_is_bit_exact(cuda):
    """p = bf16_RNE(w); rem = bf16_RNE(w - p) (sol_modules.py:423-424) for the same fp32 w.

    With lr = 0 and no decay, AdamW leaves w unchanged, so one pass of the
    kernel must reproduce torch's split of the reconstructed weight bit for bit."""
    g = torch.Generator().manual_seed(2)
    w = torch.randn(4099, generator=g) * 0.05
    p0 = w.to(torch.bfloat16)
    r0 = (w - p0.float()).to(torch.bfloat16)
    p = torch.nn.Parameter(p0.clone().cuda())
    opt = AdamW([p], lr=0.0, weight_decay=0.0, master="bf16_mt")
    p.grad = torch.zeros_like(p)
    opt._init_state(p)
    opt.state[p]["mant_rem"].copy_(r0.cuda())
    opt.step()
    torch.cuda.synchronize()
    wr = p0.float() + r0.float()
    pe = wr.to(torch.bfloat16)
    re = (wr - pe.float()).to(torch.bfloat16)
    assert torch.equal(p.data.cpu().view(torch.int16), pe.view(torch.int16))
    assert torch.equal(opt.state[p]["mant_rem"].cpu().view(torch.int16), re.view(torch.int16))


# ----------------------------------------------------------------- NorMuon --
def _normuon_pair(cfg, steps, cautious, bf16_master, orthogonalizer, coefficients="quintic", wd=0.1,
                  nesterov=True, ortho=None, engine_cls=None):
    model_c = synth.SyntheticLM(cfg, seed=0)
    model_g = synth.SyntheticLM(cfg, seed=0).cuda()
    muon_c = [p for n, p in model_c.named_parameters() if n in ref_step.route(model_c.named_parameters())[0]]
    names = ref_step.route(model_c.named_parameters())[0]
    gmap = dict(model_g.named_parameters())
    muon_g = [gmap[n] for n in names]
    orc = ref_step.RefNorMuon(muon_c, lr=8e-3, weight_decay=wd, cautious_wd=cautious, bf16_master=bf16_master,
                              nesterov=nesterov, ortho=ortho)
    eng = (engine_cls or NorMuonGNS)(muon_g, lr=8e-3, weight_decay=wd, cautious_wd=cautious,
                                     bf16_master=bf16_master, nesterov=nesterov, orthogonalizer=orthogonalizer,
                                     coefficients=coefficients)
    p0 = [p.detach().clone().float() for p in muon_c]
    for it in range(steps):
        mom = 0.85 + 0.10 * min(1.0, it / 300)
        orc.group["momentum"] = mom
        eng.param_groups[0]["momentum"] = mom
        grads = synth.make_grads(model_c, it, seed=3)
        gl = dict(zip([n for n, _ in model_c.named_parameters()], grads))
        for n, p in zip(names, muon_c):
            p.grad = gl[n]
        for n, p in zip(names, muon_g):
            p.grad = gl[n].cuda()
        orc.step()
        eng.step()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return names, muon_c, muon_g, p0, orc, eng


@pytest.mark.parametrize("cfg,cautious,mt,bound", [(synth.C1, False, False, 1e-2), (synth.MICRO, True, True, 1.5e-2),
                                                    (synth.MICRO, False, False, 2.5e-2)])
def test_normuon_quintic_matches_reference(cuda, cfg, cautious, mt, bound):
    names, pc, pg, p0, orc, eng = _normuon_pair(cfg, 10, cautious, mt, "quintic")
    du_c = torch.cat([(p.detach().float() - a).reshape(-1) for p, a in zip(pc, p0)])
    du_g = torch.cat([(p.detach().float().cpu() - a).reshape(-1) for p, a in zip(pg, p0)])
    err = rel_fro(du_g, du_c)
    print(f"{cfg.name}: cumulative update rel. Frobenius error after 10 steps = {err:.2e}")
    assert err <= bound
    for i, (a, b) in enumerate(zip(pc, pg)):
        e = rel_fro(b.detach().float().cpu() - p0[i], a.detach().float() - p0[i])
        assert e <= 3e-2, f"{names[i]}: per-matrix update error {e:.3e}"
        st_o, st_e = orc.state[i], eng.state[b]
        # the momentum buffer does not depend on the orthogonaliser: same lerps
        if a.dtype == torch.float32:
            assert_f32_ulps(st_e["momentum_buffer"], st_o["momentum_buffer"], ulps=2, what="momentum")
        else:
            assert_bf16_close(st_e["momentum_buffer"], st_o["momentum_buffer"], "momentum", min_exact=0.99)
        assert rel_fro(st_e["v_row"], st_o["v_row"]) < 3e-2


def test_normuon_gram_quintic_table_matches_reference(cuda):
    """Gram Newton-Schulz with the quintic table equals standard NS in exact
    arithmetic; the engine runs it in binary16, the reference in bf16."""
    names, pc, pg, p0, orc, eng = _normuon_pair(synth.MICRO, 10, True, True, "gram", "quintic")
    du_c = torch.cat([(p.detach().float() - a).reshape(-1) for p, a in zip(pc, p0)])
    du_g = torch.cat([(p.detach().float().cpu() - a).reshape(-1) for p, a in zip(pg, p0)])
    err = rel_fro(du_g, du_c)
    print(f"gram/quintic: cumulative update rel. Frobenius error after 10 steps = {err:.2e}")
    assert err <= 2.5e-2


@pytest.mark.parametrize("r,c", [(384, 128), (128, 384), (512, 512), (3072, 1024)])
def test_gram_binary16_is_closer_to_exact_than_reference(cuda, r, c):
    """On one orthogonalisation, the engine's binary16 Gram iteration (quintic
    table) is nearer to exact-arithmetic Newton-Schulz than the reference's own
    bf16 iteration is."""
    g = torch.Generator().manual_seed(r * 3 + c)
    U = (torch.randn(2, r, c, generator=g) * 1e-3).to(torch.bfloat16)
    opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(r, c, device=cuda))], orthogonalizer="gram",
                     coefficients="quintic")
    out = opt._orthogonalize_batch(U.cuda(), 5).float().cpu()
    exact = gram_ns_ref.gram_ns(U, [polar_express.QUINTIC] * 5)
    ref_bf16 = ref_step.ortho_batch_quintic(U, 5).float()
    e_eng, e_ref = rel_fro(out, exact), rel_fro(ref_bf16, exact)
    print(f"({r},{c}) vs exact NS: engine gram/binary16 {e_eng:.2e}, reference bf16 {e_ref:.2e}")
    assert e_eng < 1e-2 and e_eng < e_ref


@pytest.mark.parametrize("r,c", [(256, 256), (768, 256), (256, 1408), (1024, 1024), (8, 128)])
def test_gram_polar_express_vs_fp64_restatement(cuda, r, c):
    g = torch.Generator().manual_seed(r + c)
    U = (torch.randn(3, r, c, generator=g) * 1e-3).to(torch.bfloat16)
    opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(r, c, device=cuda))], orthogonalizer="gram",
                     coefficients="polar_express")
    out = opt._orthogonalize_batch(U.cuda(), 5)
    torch.cuda.synchronize()
    table = polar_express.polar_express(5)
    ref64 = gram_ns_ref.gram_ns(U, table, safety=opt.norm_safety)
    emu16 = gram_ns_ref.gram_ns(U, table, safety=opt.norm_safety, store=torch.float16)
    err, err_emu = rel_fro(out.float(), ref64), rel_fro(emu16, ref64)
    print(f"({r},{c}) gram/PE binary16 engine vs fp64: {err:.3e} (CPU binary16 emulation: {err_emu:.3e})")
    assert err < max(3e-2, 2.5 * err_emu)
    pf = gram_ns_ref.polar_factor(U)
    assert rel_fro(out.float(), pf) < 0.25


# -------------------------------------------------------------- full step --
def test_full_step_with_ema_matches_reference(cuda):
    """build_optimizers + EmaWeights (EMA folded into the passes) vs the reference
    step muon -> adamw -> ema (oracle/ref_step.RefStep, bit-exact with the
    reference on the CPU) run with torch on the same GPU: torch's CUDA fused
    AdamW and bf16 cuBLAS Newton-Schulz, 6 steps of the MICRO recipe set."""
    cfg = synth.MICRO
    kw = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)
    mr = synth.SyntheticLM(cfg, seed=0).cuda()
    mg = synth.SyntheticLM(cfg, seed=0).cuda()
    ref = ref_step.RefStep(mr, **kw)
    muon, adamw = build_optimizers(mg, orthogonalizer="quintic", **kw)
    ema = EmaWeights(mg, 0.999)
    p0 = [p.detach().clone().float() for p in mr.parameters()]
    for it in range(6):
        frac = (it + 1) / 5
        ref.muon.group["lr"] = ref.muon.group["base_lr"] * frac
        for gg in ref.adamw.param_groups:
            gg["lr"] = gg["base_lr"] * frac
        for opt in (muon, adamw):
            for gg in opt.param_groups:
                gg["lr"] = gg["base_lr"] * frac
        grads = synth.make_grads(mr, it, seed=0)
        synth.set_grads(mr, grads)
        synth.set_grads(mg, [x.clone() for x in grads])
        ref.step()
        muon.step()
        adamw.step()
        ema.update()
    torch.cuda.synchronize()
    assert ema._armed and ema._folded == set()
    named_r = list(mr.named_parameters())
    named_g = dict(mg.named_parameters())
    muon_names = set(ref_step.route(named_r)[0])
    num = den = 0.0
    for i, (n, pr) in enumerate(named_r):
        pgpu = named_g[n]
        if n in muon_names:
            du_g, du_r = pgpu.detach().float() - p0[i], pr.detach().float() - p0[i]
            num += float((du_g - du_r).pow(2).sum())
            den += float(du_r.pow(2).sum())
            assert rel_fro(ema.shadow[i] - p0[i], ref.shadow[i] - p0[i]) < 3e-2
        else:
            # AdamW: torch's CUDA fused formula, reproduced bit for bit
            assert torch.equal(pgpu.data, pr.data), n
            ms, mo = adamw.state[pgpu], ref.adamw.state[pr]
            assert torch.equal(ms["exp_avg"], mo["exp_avg"]) and torch.equal(ms["exp_avg_sq"], mo["exp_avg_sq"]), n
            # EMA of identical parameters: torch's lerp formula in fp32
            assert_f32_ulps(ema.shadow[i], ref.shadow[i], ulps=2, what=f"ema {n}")
    err = (num / den) ** 0.5
    print(f"full step: NorMuon cumulative update rel. Frobenius error after 6 steps = {err:.2e}")
    # quintic mode restates the reference's bf16 iteration rounding for rounding;
    # against the reference run with torch on the same GPU only the fp32
    # accumulation order inside the GEMMs differs (measured 9.2e-5)
    assert err < 1e-3


def test_ema_folded_equals_standalone(cuda):
    cfg = synth.MICRO
    m1 = synth.SyntheticLM(cfg, seed=0).cuda()
    m2 = synth.SyntheticLM(cfg, seed=0).cuda()
    kw = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)
    o1 = build_optimizers(m1, **kw)
    o2 = build_optimizers(m2, **kw)
    e1 = EmaWeights(m1, 0.99)
    e2 = EmaWeights(m2, 0.99, fuse=False)
    for it in range(4):
        grads = synth.make_grads(m1, it, seed=5)
        synth.set_grads(m1, grads)
        synth.set_grads(m2, [x.clone() for x in grads])
        for o in o1:
            o.step()
        e1.update()
        for o in o2:
            o.step()
        e2.update()
    torch.cuda.synchronize()
    for a, b in zip(e1.shadow, e2.shadow):
        assert_f32_ulps(a, b, ulps=0, what="ema")
    # averaged(): params become bf16(shadow) and are restored afterwards
    before = [p.detach().clone() for p in m1.parameters()]
    with e1.averaged():
        for p, s in zip(m1.parameters(), e1.shadow):
            assert torch.equal(p.data, s.to(p.dtype))
    for p, b in zip(m1.parameters(), before):
        assert torch.equal(p.data, b)


@pytest.mark.parametrize("r,c", [(8, 1024), (1024, 8), (32, 1536), (12, 4096), (33, 1024)])
def test_gram_small_matrices_match_binary16_emulation(cuda, r, c):
    """Matrices with min(r, c) <= 32 and at most 49152 elements run the whole
    iteration in one CTA per matrix (the recipe's 8 x 1024 attention gates);
    (33, 1024) takes the GEMM path. Both follow the CPU binary16 emulation of
    the same schedule up to fp32 accumulation order."""
    g = torch.Generator().manual_seed(7 * r + c)
    U = (torch.randn(5, r, c, generator=g) * 1e-3).to(torch.bfloat16)
    opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(r, c, device=cuda))], orthogonalizer="gram",
                     coefficients="polar_express")
    out = opt._orthogonalize_batch(U.cuda(), 5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    table = polar_express.polar_express(5)
    emu16 = gram_ns_ref.gram_ns(U, table, safety=opt.norm_safety, store=torch.float16)
    ref64 = gram_ns_ref.gram_ns(U, table, safety=opt.norm_safety)
    err, err64 = rel_fro(out.float(), emu16), rel_fro(out.float(), ref64)
    print(f"({r},{c}) engine vs binary16 emulation {err:.2e}, vs fp64 {err64:.2e}")
    assert err < 1e-2
    assert err64 < 3e-2


def test_multi_group_orthogonalisation_equals_per_group(cuda):
    """Shape groups sharing m = min(r, c) go through one call, whose per-group
    Gram and Q X products run as grouped GEMM launches (CTA-pair tiles here);
    grouping changes launch granularity only, so each group's result must be
    bit-identical to the group orthogonalised alone."""
    lib = _lib.load()
    shapes = [(3, 768, 256), (2, 256, 256), (2, 256, 1280), (1, 1024, 256)]
    opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(4, 4, device=cuda))], orthogonalizer="gram")
    coeffs, resets, nres = opt._table(5)
    g = torch.Generator(device=cuda).manual_seed(11)
    data = []
    for S, r, c in shapes:
        U = (torch.randn(S, r, c, generator=g, device=cuda) * 1e-3).to(torch.bfloat16)
        nparts = lib.b2o_normuon_front_parts(r * c)
        part = torch.zeros(S, nparts, device=cuda)
        part[:, 0] = U.float().pow(2).sum(dim=(1, 2))
        ntn = (c + 255) // 256
        data.append((U, part, S, r, c, ntn))

    def run(members):
        groups = (_lib.OrthoGroup * len(members))()
        outs = []
        for i, (U, part, S, r, c, ntn) in enumerate(members):
            o = torch.empty_like(U)
            rs = torch.zeros(S * ntn * r, device=cuda)
            outs.append((o, rs))
            groups[i] = _lib.OrthoGroup(U.data_ptr(), part.data_ptr(), o.data_ptr(), rs.data_ptr(), S, r, c, 0)
        nbytes = lib.b2o_ortho_workspace_bytes_multi(groups, len(members))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
        rc = lib.b2o_orthogonalize_multi(groups, len(members), 1, coeffs, 5, resets, nres, opt.norm_eps,
                                         opt.norm_safety, ws.data_ptr(), nbytes, _lib.stream_ptr())
        _lib.check(rc, "orthogonalize_multi")
        torch.cuda.synchronize()
        return outs

    together = run(data)
    assert _lib.device_error() == 0
    for i, d in enumerate(data):
        (o1, rs1), = run([d])
        o, rs = together[i]
        assert torch.equal(o, o1), f"group {d[2:5]}: output differs when grouped"
        assert torch.equal(rs, rs1), f"group {d[2:5]}: row sums differ when grouped"


# -------------------------------------------------------- gradient clip --
@pytest.mark.parametrize("max_norm", [1e-3, 1e3])
def test_clip_grad_norm_matches_torch(cuda, max_norm):
    """sol_b200.clip_grad_norm_ vs torch.nn.utils.clip_grad_norm_(foreach=True)
    (train_sol.py:498-499) on the recipe's bf16 gradients, clipping (1e-3) and
    not (1e3): the returned norm and the clipped gradients are bit-identical."""
    from sol_b200 import clip_grad_norm_
    model = synth.SyntheticLM(synth.MICRO, device=cuda, seed=0)
    grads = synth.make_grads(model, 0, seed=0)
    params = [p for _, p in model.named_parameters()]
    for p, g in zip(params, grads):
        p.grad = g.clone()
    ref = torch.nn.utils.clip_grad_norm_(params, max_norm, foreach=True)
    ref_grads = [p.grad.clone() for p in params]
    for p, g in zip(params, grads):
        p.grad = g.clone()
    got = clip_grad_norm_(params, max_norm, foreach=True)
    torch.cuda.synchronize()
    assert got.dtype == ref.dtype and float(got) == float(ref), (float(got), float(ref))
    for p, r in zip(params, ref_grads):
        assert torch.equal(p.grad, r)


def test_deferred_clip_step_equals_eager_clip_step(cuda):
    """Clipping deferred into the optimizers' passes gives the same step as
    clipping the gradients in place first."""
    from sol_b200 import clip_grad_norm_

    def run(defer):
        model = synth.SyntheticLM(synth.MICRO, device=cuda, seed=0)
        muon, adamw = build_optimizers(model, adam_master="bf16_mt", muon_lr=8e-3, adam_lr=1.2e-2,
                                       embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)
        params = [p for _, p in model.named_parameters()]
        for k in range(3):
            synth.set_grads(model, synth.make_grads(model, k, seed=0))
            clip_grad_norm_(params, 2e-3, defer_to=(muon, adamw) if defer else None)
            muon.step()
            adamw.step()
        torch.cuda.synchronize()
        return [p.detach().clone() for p in params]

    for a, b in zip(run(False), run(True)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("factor", [2.0 ** 12, 2.0 ** -12, 2.0])
def test_prescaled_x0_repair(cuda, factor):
    """The front writes the Gram input as binary16(bf16(u) * k) with k from the
    previous step's norm. Corrupting the stored k after the first step (2^12:
    X0 would overflow binary16; 2^-12: it would flush to zero; 2: still in
    range) must not change the next steps beyond rounding: out-of-range
    matrices are rewritten with this step's k before the Gram products."""
    def run(corrupt):
        model = synth.SyntheticLM(synth.MICRO, device=cuda, seed=0)
        muon, adamw = build_optimizers(model, muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1,
                                       cautious_wd=True, bf16_master=True)
        for k in range(3):
            synth.set_grads(model, synth.make_grads(model, k, seed=0))
            muon.step()
            if k == 0 and corrupt:
                for ws in muon._ws.values():
                    ws["prescale"].mul_(factor)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        return [p.detach().float().clone() for p in muon.param_groups[0]["params"]], muon

    ref, _ = run(False)
    got, muon = run(True)
    for a, b in zip(ref, got):
        assert torch.isfinite(b).all()
        assert rel_fro(b, a) < 1e-3
    if factor != 2.0:  # the corrupted batches were flagged and rewritten at step 1
        assert any(int(ws["flags"].sum()) == 0 for ws in muon._ws.values())  # step 2 needed no repair


def test_clip_grad_norm_fp32_gradients(cuda):
    """fp32 gradients (config C1): norms and coefficient in fp32, where the
    summation order may differ from torch's in the last bits."""
    from sol_b200 import clip_grad_norm_
    model = synth.SyntheticLM(synth.C1, device=cuda, seed=0)
    grads = synth.make_grads(model, 0, seed=0)
    params = [p for _, p in model.named_parameters()]
    for p, g in zip(params, grads):
        p.grad = g.clone()
    ref = torch.nn.utils.clip_grad_norm_(params, 1e-3, foreach=True)
    ref_grads = [p.grad.clone() for p in params]
    for p, g in zip(params, grads):
        p.grad = g.clone()
    got = clip_grad_norm_(params, 1e-3)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    assert abs(float(got) - float(ref)) <= 4e-7 * float(ref)
    for p, r in zip(params, ref_grads):
        assert torch.allclose(p.grad, r, rtol=4e-7, atol=0)



def _cumulative_error(pc, pg, p0):
    du_c = torch.cat([(p.detach().float() - a).reshape(-1) for p, a in zip(pc, p0)])
    du_g = torch.cat([(p.detach().float().cpu() - a).reshape(-1) for p, a in zip(pg, p0)])
    return rel_fro(du_g, du_c)


def test_normuon_without_nesterov_or_weight_decay(cuda):
    """nesterov=False (u = buf, sol_modules.py:394) and weight_decay=0 (no decay
    factor at all) against the oracle, fp32 C1, quintic mode."""
    names, pc, pg, p0, orc, eng = _normuon_pair(synth.C1, 10, False, False, "quintic", wd=0.0, nesterov=False)
    err = _cumulative_error(pc, pg, p0)
    print(f"no nesterov, no wd: cumulative update rel. Frobenius error = {err:.2e}")
    assert err <= 1e-2


def test_normuon_gram_path_vs_fp64_gram_oracle(cuda):
    """The production path (Gram Newton-Schulz, Polar Express table, binary16,
    prescaled input written by the front) on fp32 parameters against the
    oracle's NorMuon step with the fp64 Gram restatement as orthogonaliser."""
    table = polar_express.polar_express(5)

    def gram64(U, ns_steps):
        return gram_ns_ref.gram_ns(U, table).to(torch.bfloat16)

    names, pc, pg, p0, orc, eng = _normuon_pair(synth.C1, 10, True, False, "gram", "polar_express", ortho=gram64)
    err = _cumulative_error(pc, pg, p0)
    print(f"gram/PE engine vs fp64 Gram oracle step: cumulative update rel. Frobenius error = {err:.2e}")
    assert err <= 1e-2  # measured 4.3e-3 (binary16 iteration, bf16 input rounding)


def test_overridden_orthogonalizer_hook_is_used(cuda):
    """A subclass overriding _orthogonalize_batch (the reference's benches patch
    it, scripts/muon_copy_bench.py:84-89) gets the bf16 front output and its
    result drives the update: with the oracle's own quintic as the hook, the
    engine's step follows the oracle's to the apply arithmetic's rounding."""
    class Hooked(NorMuonGNS):
        calls = 0

        def _orthogonalize_batch(self, U, ns_steps):
            Hooked.calls += 1
            assert U.dtype == torch.bfloat16 and U.is_cuda
            return ref_step.ortho_batch_quintic(U.cpu(), ns_steps).to(U.device)

    names, pc, pg, p0, orc, eng = _normuon_pair(synth.C1, 5, False, False, "gram", engine_cls=Hooked)
    assert Hooked.calls > 0
    err = _cumulative_error(pc, pg, p0)
    print(f"hooked quintic vs oracle: cumulative update rel. Frobenius error = {err:.2e}")
    assert err <= 1e-3


@pytest.mark.parametrize("mode", ["quintic", "gram"])
def test_normuon_ragged_shapes_and_batch_split(cuda, mode):
    """70 same-shape matrices (batches of 64 + 6), odd shapes that take the
    scalar and CUDA-core paths, a 5 x 300 matrix (small-matrix path) and a
    parameter without gradient (skipped, sol_modules.py:378-379), against the
    oracle's step (quintic, or the fp64 Gram restatement for gram mode)."""
    g = torch.Generator().manual_seed(5)
    shapes = [(24, 40)] * 70 + [(97, 61)] * 3 + [(61, 97)] * 2 + [(5, 300)] + [(33, 33)]
    base = [torch.randn(s, generator=g) * 0.02 for s in shapes]
    pc = [torch.nn.Parameter(b.clone()) for b in base]
    pg = [torch.nn.Parameter(b.clone().cuda()) for b in base]
    table = polar_express.polar_express(5)
    ortho = (lambda U, ns: gram_ns_ref.gram_ns(U, table).to(torch.bfloat16)) if mode == "gram" else None
    orc = ref_step.RefNorMuon(pc, lr=8e-3, weight_decay=0.1, cautious_wd=True, ortho=ortho)
    eng = NorMuonGNS(pg, lr=8e-3, weight_decay=0.1, cautious_wd=True, orthogonalizer=mode,
                     coefficients="polar_express" if mode == "gram" else "quintic")
    for it in range(3):
        for i, (a, b) in enumerate(zip(pc, pg)):
            if i == len(shapes) - 1:  # the last parameter never gets a gradient
                a.grad = b.grad = None
                continue
            gr = torch.randn(a.shape, generator=g) * 1e-3
            a.grad = gr
            b.grad = gr.cuda()
        orc.step()
        eng.step()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(pg[-1].detach().cpu(), base[-1])  # no gradient: untouched
    assert "momentum_buffer" not in eng.state.get(pg[-1], {})
    err = _cumulative_error(pc[:-1], pg[:-1], base[:-1])
    print(f"{mode}: ragged/split cumulative update rel. Frobenius error = {err:.2e}")
    assert err <= 1e-2
