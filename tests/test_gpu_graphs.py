"""Launch graphs of the orthogonaliser: replaying a captured call must equal
launching its kernels directly, bit for bit, and launch the same kernels.

The engine captures the second orthogonaliser call with a given argument set
(workspace, groups, coefficients, restarts) into a CUDA graph and replays it
from the third call on. These tests step two optimizers over identical
parameters and gradients, one with graphs off and one with graphs on, and
compare every parameter and state tensor with torch.equal.
"""
import pytest
import torch

from sol_b200 import NorMuonGNS, _lib

pytestmark = pytest.mark.gpu

# one m = 256 class of three shapes (forked group streams inside the graph),
# one m = 8 class (the small-matrix kernel) and a square m = 128 class
SHAPES = [(256, 768)] * 3 + [(768, 256)] * 2 + [(256, 256)] * 2 + [(8, 256)] * 2 + [(128, 128)] * 3


def _run(cuda, mode, graphs, steps, dtype):
    g = torch.Generator(device=cuda).manual_seed(3)
    params = [torch.nn.Parameter((torch.randn(s, generator=g, device=cuda) * 0.02).to(dtype)) for s in SHAPES]
    grads = [[(torch.randn(s, generator=g, device=cuda) * 1e-3).to(dtype) for s in SHAPES] for _ in range(steps)]
    opt = NorMuonGNS(params, lr=8e-3, weight_decay=0.1, cautious_wd=True, bf16_master=dtype == torch.bfloat16,
                     orthogonalizer=mode, coefficients="polar_express" if mode == "gram" else "quintic")
    prev = _lib.launch_graphs(graphs)
    launches = []
    try:
        for k in range(steps):
            for p, gr in zip(params, grads[k]):
                p.grad = gr
            n0 = _lib.launch_count()
            opt.step()
            launches.append(_lib.launch_count() - n0)
        torch.cuda.synchronize()
    finally:
        _lib.launch_graphs(prev)
    assert _lib.device_error() == 0
    state = [{k: v.clone() for k, v in opt.state[p].items() if torch.is_tensor(v)} for p in params]
    return [p.detach().clone() for p in params], state, launches


@pytest.mark.parametrize("mode,dtype", [("gram", torch.bfloat16), ("gram", torch.float32),
                                        ("quintic", torch.bfloat16)])
def test_graph_replay_equals_direct_launches(cuda, mode, dtype):
    steps = 5  # step 1 launches directly, step 2 captures and replays, steps 3-5 replay
    s0 = _lib.launch_graph_stats()
    p_direct, st_direct, n_direct = _run(cuda, mode, False, steps, dtype)
    s1 = _lib.launch_graph_stats()
    assert s1 == s0, "graphs were used while turned off"
    p_graph, st_graph, n_graph = _run(cuda, mode, True, steps, dtype)
    s2 = _lib.launch_graph_stats()
    assert s2["failures"] == s1["failures"], "a launch-graph capture failed on this device"
    # three m-classes are orthogonalised per step: each captured once, replayed from step 2 on
    assert s2["captures"] - s1["captures"] == 3
    assert s2["replays"] - s1["replays"] == 3 * (steps - 1)
    assert n_graph == n_direct, f"kernel launches per step differ: {n_graph} vs {n_direct}"
    for i, (a, b) in enumerate(zip(p_direct, p_graph)):
        assert torch.equal(a, b), f"parameter {i} {tuple(a.shape)} differs under graph replay"
    for i, (a, b) in enumerate(zip(st_direct, st_graph)):
        assert a.keys() == b.keys()
        for k in a:
            assert torch.equal(a[k], b[k]), f"state {k} of parameter {i} differs under graph replay"


def test_changed_workspace_gets_its_own_graph(cuda):
    """A new argument set (here: a fresh workspace for the same groups) never
    replays another set's graph: its first call launches directly."""
    lib = _lib.load()
    opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(4, 4, device=cuda))], orthogonalizer="gram")
    coeffs, resets, nres = opt._table(5)
    g = torch.Generator(device=cuda).manual_seed(7)
    S, r, c = 4, 256, 512
    U = (torch.randn(S, r, c, generator=g, device=cuda) * 1e-3).to(torch.bfloat16)
    part = torch.zeros(S, lib.b2o_normuon_front_parts(r * c), device=cuda)
    part[:, 0] = U.float().pow(2).sum(dim=(1, 2))
    ntn = (c + 255) // 256
    outs = []

    def call(ws, o, rs):
        groups = (_lib.OrthoGroup * 1)()
        groups[0] = _lib.OrthoGroup(U.data_ptr(), part.data_ptr(), o.data_ptr(), rs.data_ptr(), S, r, c, 0)
        rc = lib.b2o_orthogonalize_multi(groups, 1, 1, coeffs, 5, resets, nres, opt.norm_eps, opt.norm_safety,
                                         ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        _lib.check(rc, "orthogonalize_multi")

    groups = (_lib.OrthoGroup * 1)()
    groups[0] = _lib.OrthoGroup(U.data_ptr(), part.data_ptr(), U.data_ptr(), part.data_ptr(), S, r, c, 0)
    nbytes = lib.b2o_ortho_workspace_bytes_multi(groups, 1)
    wss = [torch.empty(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
    prev = _lib.launch_graphs(True)
    try:
        for ws in wss:
            o, rs = torch.empty_like(U), torch.zeros(S * ntn * r, device=cuda)
            s0 = _lib.launch_graph_stats()
            for _ in range(3):
                call(ws, o, rs)
            s1 = _lib.launch_graph_stats()
            assert s1["captures"] - s0["captures"] == 1 and s1["replays"] - s0["replays"] == 2
            outs.append((o, rs))
        torch.cuda.synchronize()
    finally:
        _lib.launch_graphs(prev)
    assert _lib.device_error() == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_changed_iteration_count_captures_new_graphs(cuda):
    """ns_steps changed between steps (a different coefficient table and
    restart list) is a new argument set: it launches directly once, is
    captured, and the results equal direct launches throughout."""
    def run(graphs):
        g = torch.Generator(device=cuda).manual_seed(9)
        params = [torch.nn.Parameter((torch.randn(s, generator=g, device=cuda) * 0.02).to(torch.bfloat16))
                  for s in SHAPES]
        opt = NorMuonGNS(params, lr=8e-3, weight_decay=0.1, cautious_wd=True, bf16_master=True)
        prev = _lib.launch_graphs(graphs)
        try:
            for k in range(6):
                opt.param_groups[0]["ns_steps"] = 5 if k < 3 else 3
                for p in params:
                    p.grad = (torch.randn(p.shape, generator=g, device=cuda) * 1e-3).to(torch.bfloat16)
                opt.step()
            torch.cuda.synchronize()
        finally:
            _lib.launch_graphs(prev)
        assert _lib.device_error() == 0
        return [p.detach().clone() for p in params]

    direct = run(False)
    s0 = _lib.launch_graph_stats()
    graphed = run(True)
    s1 = _lib.launch_graph_stats()
    assert s1["failures"] == s0["failures"]
    assert s1["captures"] - s0["captures"] == 6  # three m-classes x two iteration counts
    assert s1["replays"] - s0["replays"] == 12
    for i, (a, b) in enumerate(zip(direct, graphed)):
        assert torch.equal(a, b), f"parameter {i} differs under graph replay"
