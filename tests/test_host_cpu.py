"""Host-side logic that needs no GPU: routing, coefficient tables, the C ABI
library's exports, and the no-CPU-fallback rule."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from oracle import gram_ns_ref, ref_step
from sol_b200 import _lib, polar_express, synth
from sol_b200.routing import route_params

ROOT = Path(__file__).resolve().parents[1]


# ------------------------------------------------------------------ routing --
@pytest.mark.parametrize("cfg", [synth.C1, synth.MICRO, synth.C2, synth.C5])
def test_routing_matches_reference(cfg):
    model = synth.SyntheticLM(cfg, device="meta")
    named = list(model.named_parameters())
    ours = route_params(named)
    ids = {id(p): n for n, p in named}
    ours_names = tuple([ids[id(p)] for p in group] for group in ours)
    assert ours_names == ref_step.route(named)


def test_c2_routing_counts():
    """L14 recipe: 14 x 5 NorMuon matrices (incl. the 8x1024 attention gate),
    7 vocabulary tables (embedding, second embedding, 5 value embeddings)."""
    model = synth.SyntheticLM(synth.C2, device="meta")
    muon, embed, norm, ve = route_params(model.named_parameters())
    assert len(muon) == 14 * 5
    shapes = sorted({tuple(p.shape) for p in muon})
    assert shapes == [(8, 1024), (1024, 1024), (1024, 5632), (3072, 1024), (5632, 1024)]
    assert sum(p.numel() for p in muon) == 14 * (3072 * 1024 + 1024 * 1024 + 8 * 1024 + 2 * 5632 * 1024)
    assert sum(p.numel() for p in embed) == 2 * 32768 * 1024
    assert ve[0].shape == (5, 32768, 1024)
    assert all(p.numel() < 100_000 for p in norm)


def test_build_optimizers_groups_as_the_reference_checks_them():
    """The routing assertions of the reference's scripts/verify_ve_gates.py:58-76,
    on the engine's build_optimizers: per-head value-embedding gate weights go to
    AdamW without weight decay, the value-embedding table group uses betas
    (0.75, 0.95), and every group keeps its base_lr (sol_modules.py:480-482)."""
    from sol_b200 import build_optimizers
    model = synth.SyntheticLM(synth.MICRO, seed=0)
    muon, adamw = build_optimizers(model, muon_lr=1e-3, adam_lr=3e-3, embed_lr=6e-3, weight_decay=0.1, ve_lr=None)
    muon_ids = {id(p) for g in muon.param_groups for p in g["params"]}
    gate_w = [p for n, p in model.named_parameters() if "_ve_gate_w" in n]
    vet = {id(p) for n, p in model.named_parameters() if "value_embeds_k" in n}
    assert gate_w and not any(id(p) in muon_ids for p in gate_w)
    ve_grp = [g for g in adamw.param_groups if any(id(p) in vet for p in g["params"])]
    assert ve_grp and tuple(ve_grp[0]["betas"]) == (0.75, 0.95)
    gate_ids = {id(p) for p in gate_w}
    gate_grp = [g for g in adamw.param_groups if any(id(p) in gate_ids for p in g["params"])]
    assert gate_grp and gate_grp[0]["weight_decay"] == 0.0
    assert muon.param_groups[0]["base_lr"] == 1e-3
    assert all("base_lr" in g for g in adamw.param_groups)


# ----------------------------------------------------------- coefficients --
def test_polar_express_table_properties():
    table = polar_express.polar_express(5)
    assert len(table) == 5
    # composition maps [1e-3, 1] into a narrow band around 1 ...
    xs = [10 ** (-3 + 3 * i / 400) for i in range(401)]
    ys = [polar_express.apply_table(table, x) for x in xs]
    assert 0.8 < min(ys) and max(ys) < 1.2
    # ... much tighter than the quintic constant iteration
    yq = [polar_express.apply_table([polar_express.QUINTIC] * 5, x) for x in xs]
    assert (max(ys) - min(ys)) < 0.75 * (max(yq) - min(yq))
    # each step is centred on 1 over its (margin-widened) interval
    lo, hi = 1e-3, 1.0
    for coef in table:
        top = hi * 1.05
        pl, pu = polar_express._poly(coef, lo), polar_express._poly(coef, top)
        assert abs((pl + pu) / 2 - 1) < 1e-12
        lo, hi = pl, pu


def _scalar_gram(sig, table, store, resets=(2,)):
    """The Gram schedule on 1x1 matrices (one singular value), every product stored in `store`."""
    def rnd(v):
        return v.to(store).double() if store is not None else v
    X0 = rnd(sig)
    R, Q, X = rnd(X0 * X0), None, X0
    T = len(table)
    for t, (a, b, c) in enumerate(table):
        if t > 0 and t in resets:
            X = rnd(Q * X)
            R = rnd(X * X)
            Q = None
        P = rnd(a + b * R + c * rnd(R * R))
        Q = P if Q is None else rnd(Q * P)
        if t < T - 1 and (t + 1) not in resets:
            R = rnd(rnd(P * R) * P)
    return rnd(Q * X)


def test_polar_express_table_is_stable_in_binary16():
    """Across singular values in [2e-3, 1] the binary16 Gram iteration stays within a
    few percent of the exact composition (no divergence at interval tops)."""
    sig = torch.logspace(-2.7, 0, 4000, dtype=torch.float64)
    table = polar_express.polar_express(5)
    exact = _scalar_gram(sig, table, None)
    half = _scalar_gram(sig, table, torch.float16)
    err = ((half - exact).abs() / exact.abs())
    assert err.max() < 0.08 and err.quantile(0.99) < 0.03
    # without the safety margin the same procedure diverges somewhere
    bad = polar_express.polar_express(5, margin=0.0)
    e2 = ((_scalar_gram(sig, bad, torch.float16) - _scalar_gram(sig, bad, None)).abs() / _scalar_gram(sig, bad, None).abs())
    assert e2.max() > 1.0


def test_remez_equioscillation():
    a, b, c, E = polar_express.optimal_odd_quintic(0.1, 1.0)
    f = lambda x: 1 - (a * x + b * x ** 3 + c * x ** 5)  # noqa: E731
    xs = [0.1 + 0.9 * i / 20000 for i in range(20001)]
    worst = max(abs(f(x)) for x in xs)
    assert worst <= abs(E) * (1 + 1e-9)
    assert abs(abs(f(0.1)) - abs(E)) < 1e-12 and abs(abs(f(1.0)) - abs(E)) < 1e-12


# ------------------------------------------------------- Gram schedule math --
def test_gram_schedule_equals_standard_ns_in_exact_arithmetic():
    """With the same coefficients, the Gram iteration (with restarts) equals the
    quintic iteration X <- aX + b(XX^T)X + c(XX^T)^2 X in float64."""
    g = torch.Generator().manual_seed(0)
    U = torch.randn(3, 24, 40, generator=g, dtype=torch.float64)
    table = [polar_express.QUINTIC] * 5
    out = gram_ns_ref.gram_ns(U, table, resets=(2,), eps=0.0)
    ref = []
    for u in U:
        X = u / torch.linalg.norm(u)
        for a, b, c in table:
            A = X @ X.t()
            X = a * X + (b * A + c * A @ A) @ X
        ref.append(X)
    torch.testing.assert_close(out, torch.stack(ref), rtol=1e-9, atol=1e-11)
    # tall inputs are iterated as their transpose
    Ut = U.transpose(1, 2).contiguous()
    torch.testing.assert_close(gram_ns_ref.gram_ns(Ut, table, eps=0.0), out.transpose(1, 2), rtol=1e-9, atol=1e-11)


def test_polar_express_gram_approaches_polar_factor():
    g = torch.Generator().manual_seed(1)
    U = torch.randn(2, 32, 64, generator=g, dtype=torch.float64)
    out = gram_ns_ref.gram_ns(U, polar_express.polar_express(5), safety=1.01)
    pf = gram_ns_ref.polar_factor(U)
    s = torch.linalg.svdvals(out)
    assert s.min() > 0.6 and s.max() < 1.25
    rel = torch.linalg.norm(out - pf) / torch.linalg.norm(pf)
    assert rel < 0.2


# ------------------------------------------------------------------- C ABI --
def _header_symbols():
    text = (ROOT / "include" / "b2o.h").read_text()
    return sorted(set(re.findall(r"\b(b2o_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert set(_header_symbols()) == set(_lib.SIGNATURES)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in _header_symbols():
        assert hasattr(lib, name), name
    assert lib.b2o_version() == 1
    assert lib.b2o_normuon_front_parts(16384) == 1
    assert lib.b2o_ortho_workspace_bytes(14, 5632, 1024) > 0
    assert lib.b2o_ortho_workspace_bytes(0, 1, 1) == -1


def test_host_validation_without_gpu():
    """Invalid arguments are rejected on the host (nothing launched)."""
    lib = _lib.load()
    rc = lib.b2o_normuon_front(None, None, 0, 4, 4, 1, 0.05, 0.95, 1, None, None, None)
    assert rc < 0 and "1..64" in _lib.last_error()
    rc = lib.b2o_adamw_step(None, 0, None, 0, 1, 1, 0.0, None)
    assert rc < 0
    rc = lib.b2o_orthogonalize(None, None, 1, 4, 4, 0, None, 5, None, 0, 1e-7, 1.0, None, 0, None, None, None)
    assert rc < 0 and "bad arguments" in _lib.last_error()


def test_no_cpu_fallback():
    from sol_b200 import NorMuonGNS, AdamW, EmaWeights
    p = torch.nn.Parameter(torch.randn(16, 8))
    p.grad = torch.randn(16, 8)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        NorMuonGNS([p]).step()
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        AdamW([p]).step()
    m = torch.nn.Linear(4, 4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        EmaWeights(m).update()
    from sol_b200 import clip_grad_norm_
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        clip_grad_norm_([p], 1.0)


def test_adamw_state_dict_layout_matches_torch():
    from sol_b200 import AdamW
    params = [torch.nn.Parameter(torch.randn(4, 4))]
    ours = AdamW(params, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, fused=True)
    ref = torch.optim.AdamW(params, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, fused=True)
    assert set(ours.state_dict()["param_groups"][0]) == set(ref.state_dict()["param_groups"][0])


def test_normuon_param_group_keys_match_reference():
    from sol_b200 import NorMuonGNS
    p = torch.nn.Parameter(torch.randn(4, 4))
    keys = set(NorMuonGNS([p]).state_dict()["param_groups"][0])
    assert keys == {"lr", "momentum", "beta2", "nesterov", "ns_steps", "weight_decay", "params"}


def test_ctypes_structs_match_header_layout():
    assert ctypes.sizeof(_lib.AdamwTensor) == 6 * 8 + 8 + 4 + 4 + 8
    assert ctypes.sizeof(_lib.AdamwGroup) == 8 * 4 + 8  # 7 floats, cautious flag, grad_scale pointer
    assert ctypes.sizeof(_lib.NormuonBatch) == 4 * 4 + 14 * 8 + 2 * 4
    assert ctypes.sizeof(_lib.OrthoGroup) == 4 * 8 + 4 * 4 + 8


def test_bf16_newton_schulz_noise_floor():
    """The reference's bf16 quintic Newton-Schulz (run on the CPU, bit-exact with
    transformer_lm.sol_modules) against the same iteration with every GEMM
    accumulated in float64 before the identical bf16 rounding: only the
    accumulation order differs, yet the outputs move by several 1e-3 relative
    Frobenius. This is the floor for comparing two bf16 implementations."""
    a, b, c = ref_step.QUINTIC
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731

    def ns_f64_acc(G):
        X = G.bfloat16()
        X = X / (X.norm() + 1e-7)
        tr = G.size(0) > G.size(1)
        if tr:
            X = X.t()
        mm = lambda x, y: bf(x.double() @ y.double())  # noqa: E731
        for _ in range(5):
            A = mm(X, X.t())
            B = bf(bf(b * A.float()) + bf(c * mm(A, A).float()))
            X = bf(bf(a * X.float()) + mm(B, X).float())
        return X.t() if tr else X

    g = torch.Generator().manual_seed(0)
    errs = []
    for shape in [(384, 128), (128, 384), (256, 256), (768, 256)]:
        G = torch.randn(shape, generator=g) * 1e-3
        ref = ref_step.zeropower_ns5(G).double()
        alt = ns_f64_acc(G).double()
        errs.append((torch.linalg.norm(ref - alt) / torch.linalg.norm(ref)).item())
    assert max(errs) > 3e-3, errs


def test_every_header_symbol_has_a_ctypes_signature():
    names = set(_header_symbols())
    assert names == set(_lib.SIGNATURES), sorted(names ^ set(_lib.SIGNATURES))


def test_host_validation_of_the_newer_entry_points():
    """Multi-batch, prescale, clip and peer-exchange calls reject bad
    arguments on the host with a message (nothing launched, no GPU needed)."""
    lib = _lib.load()
    batch = (_lib.NormuonBatch * 1)()
    assert lib.b2o_normuon_front_multi(batch, 0, 1, 0.05, 0.95, 1, None, None) < 0
    assert "batches" in _lib.last_error()
    assert lib.b2o_normuon_front_multi(batch, 1, 1, 0.05, 0.95, 1, None, None) < 0  # S = 0
    assert "1..64" in _lib.last_error()
    assert lib.b2o_normuon_prescale(batch, 17, 1, 0.05, 0.95, 1, None, 1e-7, 1.0, None) < 0
    assert lib.b2o_normuon_apply_multi(batch, 1, 3, -1e-3, 0.0, 1.0, 0, 0, 0.05, 0.0, None) < 0
    assert "dtype" in _lib.last_error()
    numels = (ctypes.c_int64 * 1)(10)
    dtypes = (ctypes.c_int * 1)(5)
    ptrs = _lib.ptr_array([0])
    assert lib.b2o_clip_scratch_floats(numels, 0) == -1
    assert lib.b2o_clip_grad_norm(ptrs, numels, dtypes, 1, 1.0, None, None, None) < 0
    assert "bad tensor" in _lib.last_error() or "fp32 or bf16" in _lib.last_error()
    assert lib.b2o_clip_scale(ptrs, numels, dtypes, 2000, None, None) < 0
    assert lib.b2o_ipc_export(None, None, None) < 0
    assert lib.b2o_ipc_import(None, None) < 0
    assert lib.b2o_copy_async(None, None, None, -1, None) < 0
    assert "copy_async" in _lib.last_error()


def test_install_rebinds_the_reference_names():
    """sol_b200.install(module) puts the engine's build_optimizers, NorMuonGNS
    and EmaWeights where train_sol.py looks them up (transformer_lm.sol_modules)."""
    import types

    import sol_b200
    fake = types.ModuleType("sol_modules_stand_in")
    fake.build_optimizers = fake.NorMuonGNS = fake.EmaWeights = None
    assert sol_b200.install(fake) is fake
    assert fake.build_optimizers is sol_b200.build_optimizers
    assert fake.NorMuonGNS is sol_b200.NorMuonGNS
    assert fake.EmaWeights is sol_b200.EmaWeights
