"""The CPU oracle (oracle/wan_block.py) against golden outputs of the
reference's own model.py source (tests/golden/make_golden.py), CPU only.

Same fp32 CPU arithmetic in the same order, so the restatement must agree to
fp32 round-off (1e-5) on outputs and pool K/V, and exactly on the KV-cache
metadata (id, mask, is_pred) after every call, including id eviction.
"""
from pathlib import Path

import pytest
import torch

from oracle import wan_block as ob
from golden.make_golden import CASES, seeded_params

FIXTURES = Path(__file__).resolve().parent / "golden" / "block_cases.pt"


@pytest.fixture(scope="module")
def golden():
    return torch.load(FIXTURES, weights_only=False)


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_oracle_matches_reference(golden, ci):
    case = golden["cases"][ci]
    D, Fd, H, pool = case["dim"], case["ffn"], case["heads"], case["pool"]
    torch.manual_seed(0)
    blk = ob.WanTransformerBlock(D, Fd, H, cross_attn_norm=True, eps=1e-6).eval()
    sums = seeded_params(blk, case["seed"])
    for name, (s1, s2) in case["param_sums"].items():
        assert sums[name] == pytest.approx((s1, s2), rel=1e-12), f"weight RNG drift in {name}"
    if pool is not None:
        blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, case["calls"][0]["x"].shape[0])
    for rec in case["calls"]:
        kw = {"update_cache": rec["update"]}
        if rec["rows"] is not None:
            kw["candidate_cache_rows"] = torch.tensor(rec["rows"], dtype=torch.int64)
        with torch.no_grad():
            out = blk(rec["x"].float(), rec["ctx"].float(), rec["temb"].float(), rec["rope"], **kw)
        assert (out - rec["out"]).abs().max().item() <= 1e-5
        if pool is not None:
            c = blk.attn1.attn_caches["pos"]
            g = rec["cache"]
            assert torch.equal(c["id"], g["id"])
            assert torch.equal(c["mask"], g["mask"])
            assert torch.equal(c["is_pred"], g["is_pred"])
            if "k" in g:
                assert (c["k"][:, g["slots"]] - g["k"]).abs().max().item() <= 1e-5
                assert (c["v"][:, g["slots"]] - g["v"]).abs().max().item() <= 1e-5


def test_rope_split_and_mesh_ids():
    """44/42/42 frequency split (model.py:258-260) and action-token grid ids
    (utils.py:33-54) of the restatement."""
    r = ob.WanRotaryPosEmbed(128)
    assert (r.f_dim, r.h_dim, r.w_dim) == (44, 42, 42)
    g = ob.get_mesh_id(2, 4, 1, 7, action=True)
    assert g.shape == (4, 8)
    assert torch.all(g[1] == -1) and torch.all(g[3] == 7)
    assert torch.allclose(g[0][:4], torch.tensor([0.2, 0.4, 0.6, 0.8]))


# ------------------------------------------------ whole-model forward + scheduler
MODEL_FIX = Path(__file__).resolve().parent / "golden" / "model_cases.pt"


def test_oracle_model_matches_reference_fixture():
    """oracle.wan_model.WanTransformer3DModel (embedders, 2 blocks, output norm
    and projection) against the reference's own forward (AST-extracted,
    tests/golden/make_model_golden.py), action and latent mode."""
    import sys
    sys.path.insert(0, str(MODEL_FIX.parent))
    from make_golden import seeded_params
    from oracle import wan_model as om
    fx = torch.load(MODEL_FIX, weights_only=False)
    torch.manual_seed(0)
    cfg = dict(fx["config"])
    model = om.WanTransformer3DModel(**cfg).eval()
    sums = seeded_params(model, seed=fx["seed"])
    assert sums.keys() == fx["param_sums"].keys()
    for k, v in sums.items():
        assert abs(v[0] - fx["param_sums"][k][0]) < 1e-6 and abs(v[1] - fx["param_sums"][k][1]) < 1e-6, k
    for case in fx["cases"]:
        with torch.no_grad():
            out = model(case["inputs"], update_cache=0, action_mode=case["action_mode"])
        assert out.shape == case["out"].shape
        assert torch.allclose(out, case["out"], rtol=1e-5, atol=1e-5), (out - case["out"]).abs().max()


def test_oracle_scheduler_matches_reference_fixture():
    from oracle import wan_model as om
    fx = torch.load(MODEL_FIX, weights_only=False)
    for rec in fx["scheduler"]:
        s = om.FlowMatchScheduler(**rec["kwargs"])
        s.set_timesteps(rec["n"])
        assert torch.equal(s.sigmas, rec["sigmas"]) and torch.equal(s.timesteps, rec["timesteps"])
        for t, want in rec["steps"]:
            assert torch.equal(s.step(rec["v"], t, rec["sample"]), want)
