"""Speculative action decoding kernels (wamb_draft_forward, wamb_spec_*,
wamb_cfg_combine) and the device K2/B2 loop against the reference's own
outputs (tests/golden/spec_cases.pt, written by make_spec_golden.py from the
reference's DirectionPredictor, choose, K3/B2 scoring and RealSpeculative
loop) and the oracle (oracle/speculative.py).

Tolerances: the draft runs in fp32 with a different summation order than
torch's, so fp32 outputs agree to 1e-4 (absolute, values of order 1) and bf16
outputs to one bf16 ulp; the element maps (tree steps, commit, CFG) round as
torch's ops do and must match bit for bit; routes must match exactly.
"""
from pathlib import Path

import pytest
import torch

from oracle import speculative as osp
from wam_ops import _lib
from wam_ops import speculative as sp

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "spec_cases.pt"


@pytest.fixture(scope="module")
def gold():
    return torch.load(GOLD, weights_only=False)


def synthetic_target(states, times):
    """make_spec_golden.synthetic_target on the device."""
    s = states.float()
    t = times.float().reshape(-1, 1, 1) / 1000.
    return (torch.tanh(0.5 * s + t) - 0.25 * s * t).to(states.dtype)


def test_draft_decode_matches_reference(cuda_device, gold):
    dp = sp.DraftPredictor(gold["draft"]["state_dict"])
    c = gold["draft"]["decode"]
    out = dp.decode(c["state"].cuda(), c["previous"].cuda(), c["scalars"].cuda().contiguous())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    torch.testing.assert_close(out.cpu(), c["out"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dt", ["torch.bfloat16", "torch.float32"])
def test_draft_forward_matches_reference(cuda_device, gold, dt):
    dp = sp.DraftPredictor(gold["draft"]["state_dict"])
    c = gold["draft"]["forward"][dt]
    out = dp(c["state"].cuda(), c["previous"].cuda(), c["timestep"], c["delta"])
    assert out.dtype == c["out"].dtype and out.shape == (2, 32, 7)
    tol = 2 ** -7 if out.dtype == torch.bfloat16 else 1e-4
    torch.testing.assert_close(out.float().cpu(), c["out"].float(), rtol=tol, atol=tol)


def test_draft_batch_rows_independent(cuda_device, gold):
    """Rows of a batch are independent CTAs: a batch of 5 equals 5 single calls."""
    dp = sp.DraftPredictor(gold["draft"]["state_dict"])
    g = torch.Generator(device="cuda").manual_seed(3)
    st = torch.randn(5, 32, 7, generator=g, device="cuda").bfloat16()
    pv = torch.randn(5, 32, 7, generator=g, device="cuda").bfloat16()
    sc = torch.rand(5, 3, generator=g, device="cuda")
    out = dp.decode(st, pv, sc)
    for r in range(5):
        assert torch.equal(out[r:r + 1], dp.decode(st[r:r + 1], pv[r:r + 1], sc[r:r + 1].contiguous()))
    ref = osp.draft_decode({k: v.float() for k, v in gold["draft"]["state_dict"].items()}, st.cpu(), pv.cpu(),
                           sc.cpu())
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2 ** -7, atol=2 ** -7)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_edge_scores_and_k2b2_route(cuda_device, dtype):
    g = torch.Generator(device="cuda").manual_seed(7)
    dirs = torch.randn(6, 32, 7, generator=g, device="cuda").to(dtype)
    vals = torch.randn(7, 32, 7, generator=g, device="cuda").to(dtype)
    dr, tr = [0, 1, 2, 3, 4, 5], [0, 0, 1, 1, 2, 2]
    scales = [-0.09, -0.09, -0.12, -0.12, -0.12, -0.12]
    s = sp.edge_scores(dirs, vals, dr, tr, scales)
    ref = osp.edge_scores(dirs.cpu(), vals.cpu(), list(zip(dr, tr)), scales)
    assert s.cpu().tolist() == pytest.approx(ref, rel=1e-5)
    sl = s.cpu().tolist()
    for tau in [0.0, min(sl) - 1e-3, sorted(sl)[2], sorted(sl)[4], max(sl) + 1.0]:
        r = sp.route(s, 0, tau).cpu().tolist()
        assert tuple(r[:3]) == osp.choose(sl, tau), tau


def test_k2b2_route_ties_and_thresholds(cuda_device, gold):
    """The reference choose() cases (ties, every threshold regime), scored
    as given, through the device route kernel."""
    scores = torch.tensor([c["scores"] for c in gold["choose"]], dtype=torch.float32, device="cuda")
    for i, c in enumerate(gold["choose"]):
        r = sp.route(scores[i], 0, c["tau"]).cpu().tolist()
        assert tuple(r[:3]) == tuple(c["route"]), c


def test_k3b2_costs_and_routes_match_reference(cuda_device, gold):
    for t in gold["k3b2"]:
        draft = torch.cat((t["first"], t["second"].reshape(4, 32, 7), t["third"].reshape(8, 32, 7))).cuda()
        costs, r_greedy = sp.route_k3b2(draft, t["target"].cuda(), t["scales"], "greedy")
        _, r_global = sp.route_k3b2(draft, t["target"].cuda(), t["scales"], "global")
        ref = list(t["first_costs"]) + [x for r in t["second_costs"] for x in r] + \
            [x for r in t["third_costs"] for q in r for x in q]
        assert costs.cpu().tolist() == pytest.approx(ref, rel=1e-5)
        assert tuple(r_greedy.cpu().tolist()[1:]) == tuple(t["greedy"])
        assert tuple(r_global.cpu().tolist()[1:]) == tuple(t["global_"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_expand_commit_cfg_bitexact(cuda_device, dtype):
    lib, st = _lib.load(), _lib.stream_ptr()
    io = int(dtype == torch.float32)
    g = torch.Generator(device="cuda").manual_seed(9)
    N = 32 * 7
    tree = torch.randn(7, 32, 7, generator=g, device="cuda").to(dtype)
    dirs = torch.randn(6, 32, 7, generator=g, device="cuda").to(dtype)
    _lib.check(lib.wamb_spec_expand(tree.data_ptr(), dirs.data_ptr(), io, 2, 2, N, -0.09, tree[1].data_ptr(), st))
    _lib.check(lib.wamb_spec_expand(tree[1].data_ptr(), dirs[2].data_ptr(), io, 4, 2, N, -0.12,
                                    tree[3].data_ptr(), st))
    t = tree.cpu()
    assert torch.equal(t[1:3], osp.flow_step(dirs[0:2].cpu(), -0.09, t[0:1].expand(2, -1, -1)))
    assert torch.equal(t[3:7], osp.flow_step(dirs[2:6].cpu(), -0.12, t[1:3, None].expand(-1, 2, -1, -1)
                                             .reshape(4, 32, 7)))
    vals = torch.randn(7, 32, 7, generator=g, device="cuda").to(dtype)
    for depth, p, c in [(0, 0, 0), (1, 1, 0), (2, 1, 1), (2, 0, 1)]:
        rte = torch.tensor([depth, p, c, 0], dtype=torch.int32, device="cuda")
        tr = tree.clone()
        prev = torch.empty(1, 32, 7, dtype=dtype, device="cuda")
        _lib.check(lib.wamb_spec_commit(rte.data_ptr(), vals.data_ptr(), tr.data_ptr(), io, N, -0.09, -0.12, -0.15,
                                        tr.data_ptr(), prev.data_ptr(), st))
        sel = 0 if depth == 0 else (1 + p if depth == 1 else 3 + 2 * p + c)
        d = [-0.09, -0.12, -0.15][depth]
        assert torch.equal(tr[0].cpu(), osp.flow_step(vals[sel].cpu(), d, tree[sel].cpu()))
        assert torch.equal(prev[0], vals[sel])
    cond, unc = vals[:3], vals[3:6]
    for s in (1.0, 2.5):
        got = sp.cfg_combine(torch.cat((cond, unc)), 3, s)
        want = unc + s * (cond - unc) if s > 1 else cond
        assert torch.equal(got, want)


def test_k2b2_loop_matches_reference(cuda_device, gold):
    """The device loop against the reference RealSpeculative.loop (same
    synthetic target, the fixture's draft weights): identical rounds and a
    final state within two bf16 ulps."""
    L = gold["loop"]
    dp = sp.DraftPredictor(gold["draft"]["state_dict"])
    for run in L["runs"]:
        spec = sp.K2B2Speculative(synthetic_target, dp, run["tau"])
        final = spec.loop(L["state"].cuda(), L["timesteps"].tolist(), L["deltas"].tolist())
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        assert spec.rounds == [tuple(r) for r in run["rounds"]], run["tau"]
        torch.testing.assert_close(final.float().cpu(), run["final"].float(), rtol=2 ** -6, atol=2 ** -6)


def test_native_action_target(cuda_device):
    """NativeActionTarget on time-major candidate states equals the model's
    channel-major action forward with the same read-only candidate rows, and
    its CFG rows equal uncond + s (cond - uncond) of separate forwards."""
    sys_path = str(Path(__file__).resolve().parent)
    import sys
    if sys_path not in sys.path:
        sys.path.insert(0, sys_path)
    from test_gpu_model import _oracle_model, _to_device
    from oracle import wan_block as ob
    from wam_ops.configs import rope_freqs
    from wam_ops.model import NativeWanModel
    m = _oracle_model(seed=21)
    pool, hist, K, A = 96, 64, 3, 30
    g = torch.Generator().manual_seed(4)
    for blk in m.blocks:
        blk.attn1.init_kv_cache("pos", pool, 2, 128, "cpu", torch.float32, 2)
        c = blk.attn1.attn_caches["pos"]
        c["k"].copy_(torch.randn(c["k"].shape, generator=g))
        c["v"].copy_(torch.randn(c["v"].shape, generator=g))
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist) // 32
    dev = _to_device(m)
    for blk in dev.blocks:
        c = blk.attn1.attn_caches["pos"]
        for k in list(c):
            c[k] = c[k].to(device="cuda", dtype=torch.bfloat16 if k in ("k", "v") else c[k].dtype)
    nm = NativeWanModel(dev)
    text = torch.randn(2, 16, 64, generator=g).cuda().bfloat16()
    grid = ob.get_mesh_id(8, 4, 1, 0, action=True)
    rope = rope_freqs(grid.to(device="cuda", dtype=torch.float64))
    states = torch.randn(K, 32, A, generator=g).cuda().bfloat16()
    times = torch.tensor([900., 800., 800.], device="cuda")
    with torch.no_grad():
        nm.prepare_context(text[:1])
        got = sp.NativeActionTarget(nm, (8, 4, 1), rope)(states, times)
        x = states.permute(0, 2, 1).reshape(K, A, 8, 4, 1).contiguous()
        want = nm.forward({"noisy_latents": x, "rotary_emb": rope, "timesteps": times[:, None].expand(K, 8)
                           .contiguous()}, 0, "pos", True,
                          candidate_cache_rows=torch.zeros(K, dtype=torch.int64, device="cuda"))
        assert torch.equal(got, want)
        nm.prepare_context(text)   # [conditional, negative]
        cfg = sp.NativeActionTarget(nm, (8, 4, 1), rope, guidance_scale=3.0)(states, times)
        rows0 = torch.zeros(K, dtype=torch.int64, device="cuda")
        rows1 = torch.ones(K, dtype=torch.int64, device="cuda")
        tt = times[:, None].expand(K, 8).contiguous()
        cond = nm.forward({"noisy_latents": x, "rotary_emb": rope, "timesteps": tt}, 0, "pos", True,
                          candidate_cache_rows=rows0, context_rows=rows0)
        unc = nm.forward({"noisy_latents": x, "rotary_emb": rope, "timesteps": tt}, 0, "pos", True,
                         candidate_cache_rows=rows1, context_rows=rows1)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = unc + 3.0 * (cond - unc)
    torch.testing.assert_close(cfg.float(), ref.float(), rtol=2 ** -6, atol=2e-2)
