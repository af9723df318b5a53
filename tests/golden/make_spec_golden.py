"""Golden fixtures that pin oracle/speculative.py to the reference source.

Run in the build container, where the reference tree is mounted:
    python tests/golden/make_spec_golden.py [REFERENCE_ROOT]
It imports, as they are, the FastWAM DirectionPredictor and the K2/B2 loop
(投机采样/fastwam-base/fullcode-v1/draft.py, real_speculative.py with its
simulation_reference.py) and the K3/B2 scoring / selection
(投机采样/wam-p0-worktree/wan_va/utils/p0_k3_b2.py), runs seeded CPU cases and
writes tests/golden/spec_cases.pt:
  draft    a randomly initialised DirectionPredictor (state_dict included),
           decode() on a batch of 3 and forward() on bf16 / fp32 states
  choose   300 score vectors (ties and threshold cases included) and routes
  k3b2     16 random trees: per-edge costs and greedy / global routes
  loop     RealSpeculative.loop over 10 updates for four thresholds, with a
           deterministic synthetic target and the flow-match Euler step
           (fp32, one rounding) standing in for the scheduler
Nothing in the GPU tests, smoke() or bench.py runs this script.
"""
import importlib.util
import math
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def synthetic_target(states, times):
    """A deterministic stand-in for the target model's action directions."""
    s = states.float()
    t = times.float().reshape(-1, 1, 1) / 1000.
    return (torch.tanh(0.5 * s + t) - 0.25 * s * t).to(states.dtype)


def flow_step(v, delta, sample):
    return (sample.float() + v.float() * float(delta)).to(sample.dtype)


def main():
    root = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    fc = root / "投机采样/fastwam-base/fullcode-v1"
    sys.path.insert(0, str(fc))
    draft_mod = _load(fc / "draft.py", "ref_draft")
    spec_mod = _load(fc / "real_speculative.py", "ref_real_speculative")
    k3 = _load(root / "投机采样/wam-p0-worktree/wan_va/utils/p0_k3_b2.py", "ref_p0_k3_b2")
    g = torch.Generator().manual_seed(0)
    out = {}

    # ---------------------------------------------------------------- draft
    model = draft_mod.DirectionPredictor().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.1)
        model.feature_mean.copy_(torch.randn(451, generator=g) * 0.3)
        model.feature_std.copy_(torch.rand(451, generator=g) + 0.5)
        model.residual_mean.copy_(torch.randn(224, generator=g) * 0.05)
        model.residual_std.copy_(torch.rand(224, generator=g) * 0.2 + 0.05)
        st = torch.randn(3, 32, 7, generator=g)
        pv = torch.randn(3, 32, 7, generator=g)
        sc = torch.rand(3, 3, generator=g)
        dec = model.decode(st, pv, sc)
        fwd = {}
        for dt in (torch.bfloat16, torch.float32):
            s1 = torch.randn(1, 32, 7, generator=g).to(dt)
            p1 = torch.randn(1, 32, 7, generator=g).to(dt)
            t, d = torch.tensor(937.5), torch.tensor(-0.0625)
            fwd[str(dt)] = dict(state=s1, previous=p1, timestep=t, delta=d, out=model(s1, p1, t, d))
    out["draft"] = dict(state_dict={k: v.clone() for k, v in model.state_dict().items()},
                        decode=dict(state=st, previous=pv, scalars=sc, out=dec), forward=fwd)

    # --------------------------------------------------------------- choose
    cases = []
    for k in range(300):
        if k % 3 == 0:
            s = (torch.randint(0, 4, (6,), generator=g).float() * 0.25).tolist()   # ties
        else:
            s = (torch.rand(6, generator=g) * 2).tolist()
        tau = [0.0, 0.25, 0.5, 1.0, 1.5, 3.0][k % 6]
        cases.append(dict(scores=s, tau=tau, route=spec_mod.choose(s, tau)))
    out["choose"] = cases

    # ----------------------------------------------------------------- k3b2
    trees = []
    shp = (32, 7)
    for k in range(16):
        r = lambda *s: torch.randn(*s, *shp, generator=g)  # noqa: E731
        tree = k3.K3B2Tree(root_state=r(), root_previous_direction=r(), first_directions=r(2),
                           first_states=r(2), second_directions=r(2, 2), second_states=r(2, 2),
                           third_directions=r(2, 2, 2), third_states=r(2, 2, 2),
                           sigma_path=(1.0, 0.9, 0.75, 0.6), target_timesteps=(1000., 900., 750., 600.),
                           transition_scales=(-0.1, -0.15, -0.15))
        tgt = r(7)
        scores = k3.score_k3_b2_tree(tree, tgt)
        trees.append(dict(first=tree.first_directions, second=tree.second_directions,
                          third=tree.third_directions, target=tgt, scales=tree.transition_scales,
                          first_costs=scores.first_costs, second_costs=scores.second_costs,
                          third_costs=scores.third_costs,
                          greedy=k3.select_k3_b2_route(scores, selector="greedy"),
                          global_=k3.select_k3_b2_route(scores, selector="global")))
    out["k3b2"] = [dict(t, greedy=(t["greedy"].parent, t["greedy"].child, t["greedy"].grandchild),
                        global_=(t["global_"].parent, t["global_"].child, t["global_"].grandchild))
                   for t in trees]

    # ----------------------------------------------------------------- loop
    class Sched:
        step = staticmethod(flow_step)

    class Model:
        infer_action_scheduler = Sched()

    def fn(latents_action, timestep_action, **_):
        return synthetic_target(latents_action, timestep_action)

    ctx, mask = torch.zeros(1, 2, 4), torch.zeros(1, 2)
    cache = [torch.zeros(1, 3, 4)]
    timesteps = torch.linspace(1000., 100., 10)
    deltas = torch.full((10,), -0.09)
    state0 = torch.randn(1, 32, 7, generator=g).bfloat16()
    loops = []
    for tau in (0.0, 0.3, 0.35, 10.0):
        rs = spec_mod.RealSpeculative(Model(), model, tau)
        with torch.no_grad():
            final = rs.loop(state0.clone(), timesteps, deltas, ctx, mask, cache, cache, None, fn, False)
        loops.append(dict(tau=tau, final=final,
                          rounds=[(r["step"], r.get("depth"), r.get("parent"), r.get("child"))
                                  for r in rs.rounds]))
    out["loop"] = dict(state=state0, timesteps=timesteps, deltas=deltas, runs=loops)
    torch.save(out, HERE / "spec_cases.pt")
    print("wrote", HERE / "spec_cases.pt")


if __name__ == "__main__":
    main()
