"""oracle/speculative.py against the reference's own draft predictor, route
rules and K2/B2 loop (fixtures from tests/golden/make_spec_golden.py)."""
from pathlib import Path

import pytest
import torch

from oracle import speculative as osp

GOLD = Path(__file__).resolve().parent / "golden" / "spec_cases.pt"


@pytest.fixture(scope="module")
def gold():
    return torch.load(GOLD, weights_only=False)


def _weights(gold):
    return {k: v.float() for k, v in gold["draft"]["state_dict"].items()}


def synthetic_target(states, times):
    """The fixture script's stand-in target (make_spec_golden.synthetic_target)."""
    s = states.float()
    t = times.float().reshape(-1, 1, 1) / 1000.
    return (torch.tanh(0.5 * s + t) - 0.25 * s * t).to(states.dtype)


def test_draft_decode_matches_reference(gold):
    W, c = _weights(gold), gold["draft"]["decode"]
    assert set(W) == set(osp.DRAFT_KEYS)
    out = osp.draft_decode(W, c["state"], c["previous"], c["scalars"])
    torch.testing.assert_close(out, c["out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dt", ["torch.bfloat16", "torch.float32"])
def test_draft_forward_matches_reference(gold, dt):
    W, c = _weights(gold), gold["draft"]["forward"][dt]
    out = osp.draft_forward(W, c["state"], c["previous"], c["timestep"], c["delta"])
    assert out.dtype == c["out"].dtype and out.shape == (2, 32, 7)
    # bf16: the fp32 results agree to ~1e-6, so at most one bf16 ulp apart
    tol = 2 ** -7 if out.dtype == torch.bfloat16 else 1e-5
    torch.testing.assert_close(out.float(), c["out"].float(), rtol=tol, atol=tol)


def test_choose_matches_reference(gold):
    for c in gold["choose"]:
        assert osp.choose(c["scores"], c["tau"]) == tuple(c["route"]), c


def test_k3b2_scores_and_routes_match_reference(gold):
    for t in gold["k3b2"]:
        draft = torch.cat((t["first"], t["second"].reshape(4, 32, 7), t["third"].reshape(8, 32, 7)))
        # edges: first p vs root target 0; second (p, c) vs target 1 + p; third (p, c, g) vs 3 + 2p + c
        edges = [(p, 0) for p in range(2)] + [(2 + 2 * p + c, 1 + p) for p in range(2) for c in range(2)] + \
                [(6 + 4 * p + 2 * c + g2, 3 + 2 * p + c) for p in range(2) for c in range(2) for g2 in range(2)]
        scales = [t["scales"][0]] * 2 + [t["scales"][1]] * 4 + [t["scales"][2]] * 8
        s = osp.edge_scores(draft, t["target"], edges, scales, scale_inside=True)
        ref = list(t["first_costs"]) + [x for r in t["second_costs"] for x in r] + \
            [x for r in t["third_costs"] for q in r for x in q]
        assert s == pytest.approx(ref, rel=1e-6)
        first, second, third = t["first_costs"], t["second_costs"], t["third_costs"]
        assert osp.select_k3b2(first, second, third, "greedy") == tuple(t["greedy"])
        assert osp.select_k3b2(first, second, third, "global") == tuple(t["global_"])


def test_k2b2_loop_matches_reference(gold):
    W, L = _weights(gold), gold["loop"]
    draft = lambda s, p, t, d: osp.draft_forward(W, s, p, t, d)  # noqa: E731
    for run in L["runs"]:
        final, rounds = osp.k2b2_loop(L["state"].clone(), L["timesteps"], L["deltas"], synthetic_target, draft,
                                      run["tau"])
        assert [r[:4] for r in rounds] == [tuple(r) for r in run["rounds"]], run["tau"]
        torch.testing.assert_close(final.float(), run["final"].float(), rtol=2 ** -7, atol=2 ** -7)


def test_host_draft_scalars_match_reference_fp32():
    """The speculative loop computes the draft's (sigma, sigma + delta,
    sigma) on the host in fp32; they must equal the reference's torch fp32
    arithmetic (draft.py:38-41) bit for bit."""
    from wam_ops import speculative as sp
    g = torch.Generator().manual_seed(1)
    for t, d in zip((torch.rand(200, generator=g) * 1000).tolist(), (-torch.rand(200, generator=g) * 0.2).tolist()):
        host = torch.tensor(sp.draft_scalars(t, d), dtype=torch.float32)
        ref = osp.draft_scalars(torch.tensor(t), torch.tensor(d))[0]
        assert torch.equal(host, ref), (t, d)
