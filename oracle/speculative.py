"""CPU oracle of the speculative action-decoding pieces around the target
model -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restated from the reference:
  draft_decode / draft_forward   FastWAM DirectionPredictor
                                 (投机采样/fastwam-base/fullcode-v1/draft.py:10-42): a
                                 pre-norm TransformerEncoderLayer(64, 4 heads,
                                 FFN 256, exact GELU, LayerNorm eps 1e-5) over
                                 32 time-major positions, written out op by op
  edge_scores                    weighted L2 of draft vs target directions
                                 (real_speculative.py:75-77: norm then |delta|;
                                 p0_k3_b2.py:220-232: scale inside the norm)
  choose                         K2/B2 depth-then-cost route
                                 (real_speculative.py:13-23)
  select_k3b2                    K3/B2 greedy / global route (p0_k3_b2.py:258-283)
  flow_step                      the flow-match Euler step sample + v * delta,
                                 computed in fp32 and rounded once to the
                                 sample dtype (the product's scheduler step)
  k2b2_loop                      RealSpeculative.loop without the profiling and
                                 audit branches (real_speculative.py:32-109)

Pinned by tests/golden/make_spec_golden.py, which runs the reference's own
DirectionPredictor, choose, RealSpeculative.loop and K3/B2 scoring /
selection on seeded inputs (tests/test_oracle_speculative.py).
"""
import math

import torch
import torch.nn.functional as F

# state_dict names of the reference DirectionPredictor (draft.py:12-20).
DRAFT_KEYS = (
    "embed.weight", "embed.bias", "position",
    "block.self_attn.in_proj_weight", "block.self_attn.in_proj_bias",
    "block.self_attn.out_proj.weight", "block.self_attn.out_proj.bias",
    "block.linear1.weight", "block.linear1.bias", "block.linear2.weight", "block.linear2.bias",
    "block.norm1.weight", "block.norm1.bias", "block.norm2.weight", "block.norm2.bias",
    "head.weight", "head.bias",
    "feature_mean", "feature_std", "residual_mean", "residual_std",
)


def _encoder_layer(W, x, heads=4, eps=1e-5):
    """nn.TransformerEncoderLayer(norm_first=True, activation='gelu', dropout 0)
    in eval: x + SA(LN1(x)), then + FFN(LN2(x))."""
    b, t, e = x.shape
    hd = e // heads
    y = F.layer_norm(x, (e,), W["block.norm1.weight"], W["block.norm1.bias"], eps)
    qkv = y @ W["block.self_attn.in_proj_weight"].t() + W["block.self_attn.in_proj_bias"]
    q, k, v = qkv.split(e, -1)
    q = q.reshape(b, t, heads, hd).transpose(1, 2)
    k = k.reshape(b, t, heads, hd).transpose(1, 2)
    v = v.reshape(b, t, heads, hd).transpose(1, 2)
    p = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(hd), -1)
    o = (p @ v).transpose(1, 2).reshape(b, t, e)
    x = x + o @ W["block.self_attn.out_proj.weight"].t() + W["block.self_attn.out_proj.bias"]
    z = F.layer_norm(x, (e,), W["block.norm2.weight"], W["block.norm2.bias"], eps)
    u = F.gelu(z @ W["block.linear1.weight"].t() + W["block.linear1.bias"])
    return x + u @ W["block.linear2.weight"].t() + W["block.linear2.bias"]


def draft_decode(W, state, previous, scalars):
    """draft.py:26-36: [b, 32, A] state / previous direction and [b, 3]
    scalars -> [b, 2, 32, A] candidate directions (fp32)."""
    b, t, a = state.shape
    s = t * a
    state, previous = state.float().reshape(b, s), previous.float().reshape(b, s)
    features = torch.cat((state, previous, scalars.float()), 1)
    x = (features - W["feature_mean"]) / W["feature_std"]
    x = torch.cat((x[:, :s].reshape(b, t, a), x[:, s:2 * s].reshape(b, t, a),
                   x[:, 2 * s:, None].transpose(1, 2).expand(-1, t, -1)), -1)
    y = _encoder_layer(W, x @ W["embed.weight"].t() + W["embed.bias"] + W["position"])
    y = y @ W["head.weight"].t() + W["head.bias"]
    center, spread = y[..., :a], y[..., a:]
    residual = torch.stack((center + spread, center - spread), 1).reshape(b, 2, s)
    return (previous[:, None] + residual * W["residual_std"] + W["residual_mean"]).reshape(b, 2, t, a)


def draft_scalars(timestep, delta):
    """draft.py:38-41: (sigma, sigma + delta, sigma), sigma = timestep / 1000, fp32."""
    sigma = torch.as_tensor(timestep).float() / 1000.
    return torch.stack((sigma, sigma + torch.as_tensor(delta).float(), sigma)).reshape(1, 3)


def draft_forward(W, state, previous, timestep, delta):
    """draft.py:38-42 for one [1, 32, A] state: [2, 32, A] in state.dtype."""
    return draft_decode(W, state, previous, draft_scalars(timestep, delta)).to(state.dtype)[0]


def edge_scores(draft, target, edges, scales, scale_inside=False):
    """Per edge (d, t): ||draft[d] - target[t]|| * |scale| (fp32 norm), or
    ||(draft[d] - target[t]) * scale|| with scale_inside (p0_k3_b2.py:231)."""
    out = []
    for (d, t), s in zip(edges, scales):
        r = draft[d].float() - target[t].float()
        if scale_inside:
            out.append(float(torch.linalg.vector_norm(r * float(s))))
        else:
            out.append(float(r.flatten().norm() * torch.tensor(float(s)).abs()))
    return out


def choose(scores, tau):
    """real_speculative.py:13-23: the deepest route whose edges stay within
    tau, then the lowest cost, then the lowest (parent, child)."""
    routes = []
    for p in range(2):
        for c in range(2):
            a, b = scores[p], scores[2 + p * 2 + c]
            depth = 0 if a > tau else 1 if b > tau else 2
            routes.append((depth, a + b, p, c))
    d, _, p, c = min(routes, key=lambda r: (-r[0], r[1], r[2], r[3]))
    return d, p, c


def select_k3b2(first, second, third, selector):
    """p0_k3_b2.py:258-283 over first[2], second[2][2], third[2][2][2]."""
    if selector == "greedy":
        p = min(range(2), key=lambda i: (first[i], i))
        c = min(range(2), key=lambda i: (second[p][i], i))
        g = min(range(2), key=lambda i: (third[p][c][i], i))
        return p, c, g
    return min(((p, c, g) for p in range(2) for c in range(2) for g in range(2)),
               key=lambda r: (first[r[0]] + second[r[0]][r[1]] + third[r[0]][r[1]][r[2]], r[0], r[1], r[2]))


def flow_step(v, delta, sample):
    """sample + v * delta in fp32, rounded once to sample.dtype."""
    return (sample.float() + v.float() * float(delta)).to(sample.dtype)


def k2b2_loop(state, timesteps, deltas, target, draft, tau):
    """RealSpeculative.loop (real_speculative.py:32-109) for one [1, 32, A]
    state over len(timesteps) updates: target(states, times) -> directions,
    draft(state, previous, timestep, delta) -> [2, 32, A]. Returns the final
    state and the rounds as (step, depth, parent, child, scores)."""
    n = len(timesteps)
    i, previous, rounds = 0, None, []
    while i < n:
        if previous is None or n - i < 3:
            v = target(state, timesteps[i:i + 1])
            state = flow_step(v, deltas[i], state)
            previous = v
            rounds.append((i, None, None, None, None))
            i += 1
            continue
        dirs1 = draft(state, previous, timesteps[i], deltas[i])
        parents = flow_step(dirs1, deltas[i], state.expand(2, -1, -1))
        dirs2 = torch.stack([draft(parents[j:j + 1], dirs1[j:j + 1], timesteps[i + 1], deltas[i + 1])
                             for j in range(2)])
        shp = state.shape[1:]
        leaves = flow_step(dirs2.reshape(4, *shp), deltas[i + 1],
                           parents[:, None].expand(-1, 2, -1, -1).reshape(4, *shp))
        packed = torch.cat((state, parents, leaves), 0)
        times = torch.cat((timesteps[i:i + 1], timesteps[i + 1:i + 2].expand(2), timesteps[i + 2:i + 3].expand(4)))
        values = target(packed, times)
        first = (dirs1.float() - values[0:1].float()).flatten(1).norm(dim=1) * torch.tensor(float(deltas[i])).abs()
        second = ((dirs2.float() - values[1:3, None].float()).flatten(2).norm(dim=2)
                  * torch.tensor(float(deltas[i + 1])).abs())
        scores = torch.cat((first, second.flatten())).tolist()
        depth, parent, child = choose(scores, tau)
        if depth == 0:
            state = flow_step(values[0:1], deltas[i], state)
            previous = values[0:1]
        elif depth == 1:
            state = flow_step(values[1 + parent:2 + parent], deltas[i + 1], parents[parent:parent + 1])
            previous = values[1 + parent:2 + parent]
        else:
            leaf = 3 + 2 * parent + child
            state = flow_step(values[leaf:leaf + 1], deltas[i + 2], leaves[leaf - 3:leaf - 2])
            previous = values[leaf:leaf + 1]
        rounds.append((i, depth, parent, child, scores))
        i += depth + 1
    return state, rounds
