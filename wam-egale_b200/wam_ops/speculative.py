"""Speculative action decoding around the target model, on the device.

Mirrors the reference's K2/B2 loop (投机采样/fastwam-base/fullcode-v1/
real_speculative.py:32-109): at each round a draft predictor proposes two
directions from the current state, each is stepped to a parent state, the
draft proposes two directions from each parent, which are stepped to four
leaves; ONE batched target call evaluates the seven states (root, parents,
leaves); the weighted L2 between draft and target directions scores the six
edges; the deepest route within the threshold tau (then the cheapest) is
accepted and 1-3 updates are committed. Every piece runs in libwamb.so:

  DraftPredictor      FastWAM DirectionPredictor (fullcode-v1/draft.py:10-48),
                      wamb_draft_forward
  K2B2Speculative     the loop; tree states by wamb_spec_expand into one packed
                      [7, 32, A] buffer (no pack copy), edge scores
                      (wamb_spec_scores), route (wamb_spec_route) and commit
                      (wamb_spec_commit) on the device; the host reads the
                      4-int route once a round, as the reference reads its
                      scores (real_speculative.py:77)
  route_k3b2          the K3/B2 greedy / global selector over 14 edge costs
                      (wan_va/utils/p0_k3_b2.py:258-283)
  pack_cfg, cfg_combine   candidate rows for classifier-free guidance
                      (wan_va_server.py:747-780, 1936-1941)
  NativeActionTarget  the target: NativeWanModel in action mode over the
                      read-only KV history (candidate_cache_rows)
  GraphedTarget       a target replayed from per-batch-size CUDA graphs

The flow-match step is the product's scheduler step (sample + v * delta in
fp32, one rounding to the state dtype).
"""
import ctypes

import numpy as np
import torch

from . import _lib

ctypes_int32 = ctypes.c_int32
ctypes_float = ctypes.c_float

DRAFT_KEYS = (
    "embed.weight", "embed.bias", "position",
    "block.self_attn.in_proj_weight", "block.self_attn.in_proj_bias",
    "block.self_attn.out_proj.weight", "block.self_attn.out_proj.bias",
    "block.linear1.weight", "block.linear1.bias", "block.linear2.weight", "block.linear2.bias",
    "block.norm1.weight", "block.norm1.bias", "block.norm2.weight", "block.norm2.bias",
    "head.weight", "head.bias",
    "feature_mean", "feature_std", "residual_mean", "residual_std",
)


def _io(t):
    if t.dtype not in (torch.bfloat16, torch.float32) or not t.is_cuda:
        raise ValueError("states and directions must be CUDA bf16 or fp32 tensors")
    return int(t.dtype == torch.float32)


def draft_scalars(timestep, delta):
    """(sigma, sigma + delta, sigma), sigma = timestep / 1000, in fp32 as
    the reference computes them (draft.py:38-41)."""
    sigma = np.float32(timestep) / np.float32(1000.0)
    return [sigma, np.float32(sigma + np.float32(delta)), sigma]


class DraftPredictor:
    """Device copy of a DirectionPredictor (module or state_dict with the
    reference's names) run by wamb_draft_forward: 32 positions, width 64,
    4 heads, FFN 256, A action channels per position."""

    def __init__(self, source, device="cuda"):
        sd = source.state_dict() if hasattr(source, "state_dict") else source
        self.w = {k: sd[k].detach().to(device=device, dtype=torch.float32).contiguous() for k in DRAFT_KEYS}
        e = self.w["embed.weight"]
        if e.shape[0] != 64 or (e.shape[1] - 3) % 2 or self.w["position"].shape[-2:] != (32, 64):
            raise ValueError("unsupported draft shape (tokens 32, width 64)")
        self.channels = (e.shape[1] - 3) // 2
        if self.w["head.weight"].shape != (2 * self.channels, 64):
            raise ValueError("head width must be 2 x channels")
        p = _lib.DraftParams()
        p.tokens, p.channels, p.width, p.heads, p.ffn, p.ln_eps = 32, self.channels, 64, 4, 256, 1e-5
        names = ["embed_w", "embed_b", "position", "in_proj_w", "in_proj_b", "out_proj_w", "out_proj_b",
                 "linear1_w", "linear1_b", "linear2_w", "linear2_b", "norm1_w", "norm1_b", "norm2_w", "norm2_b",
                 "head_w", "head_b", "feature_mean", "feature_std", "residual_mean", "residual_std"]
        for n, k in zip(names, DRAFT_KEYS):
            setattr(p, n, self.w[k].data_ptr())
        self.params = p

    def decode(self, state, previous, scalars, out=None):
        """DirectionPredictor.decode (draft.py:26-36): [b, 32, A] states and
        previous directions, [b, 3] fp32 scalars -> [b, 2, 32, A]."""
        b = state.shape[0]
        if state.shape != (b, 32, self.channels) or previous.shape != state.shape or previous.dtype != state.dtype:
            raise ValueError("state / previous must be [b, 32, channels] of one dtype")
        if scalars.shape != (b, 3) or scalars.dtype != torch.float32 or not scalars.is_contiguous():
            raise ValueError("scalars must be contiguous fp32 [b, 3]")
        if out is None:
            out = torch.empty(b, 2, 32, self.channels, dtype=state.dtype, device=state.device)
        _lib.check(_lib.load().wamb_draft_forward(self.params, state.data_ptr(), previous.data_ptr(), _io(state),
                                                  scalars.data_ptr(), b, out.data_ptr(), _lib.stream_ptr()))
        return out

    def __call__(self, state, previous, timestep, delta):
        """DirectionPredictor.forward (draft.py:38-42) for one [1, 32, A] state."""
        sc = torch.tensor([draft_scalars(float(timestep), float(delta))], dtype=torch.float32,
                          device=state.device)
        return self.decode(state.contiguous(), previous.contiguous(), sc)[0]


def edge_scores(draft, target, draft_rows, target_rows, scales, scale_inside=False, out=None):
    """Weighted L2 per edge on the device (wamb_spec_scores)."""
    n = draft[0].numel()
    k = len(draft_rows)
    if out is None:
        out = torch.empty(k, dtype=torch.float32, device=draft.device)
    dr = (ctypes_int32 * k)(*draft_rows)
    tr = (ctypes_int32 * k)(*target_rows)
    sc = (ctypes_float * k)(*[float(s) for s in scales])
    _lib.check(_lib.load().wamb_spec_scores(draft.data_ptr(), target.data_ptr(), _io(draft), n, k, dr, tr, sc,
                                            int(scale_inside), out.data_ptr(), _lib.stream_ptr()))
    return out


def route(scores, mode, tau=0.0, out=None):
    """wamb_spec_route: mode 0 K2/B2 (depth, parent, child, 0); mode 1 / 2
    K3/B2 greedy / global (3, parent, child, grandchild)."""
    if out is None:
        out = torch.empty(4, dtype=torch.int32, device=scores.device)
    _lib.check(_lib.load().wamb_spec_route(scores.data_ptr(), mode, float(tau), out.data_ptr(), _lib.stream_ptr()))
    return out


def route_k3b2(draft, target, scales, selector):
    """K3/B2 scoring and route (p0_k3_b2.py:220-283): draft rows = first[2],
    second[2][2], third[2][2][2] directions, target rows = root, first[2],
    second[2][2] target directions, scales = the three transition scales.
    Returns (costs [14] fp32, route [4] int32) on the device."""
    edges = [(p, 0) for p in range(2)] + [(2 + 2 * p + c, 1 + p) for p in range(2) for c in range(2)] + \
            [(6 + 4 * p + 2 * c + g, 3 + 2 * p + c) for p in range(2) for c in range(2) for g in range(2)]
    sc = [scales[0]] * 2 + [scales[1]] * 4 + [scales[2]] * 8
    costs = edge_scores(draft, target, [e[0] for e in edges], [e[1] for e in edges], sc, scale_inside=True)
    return costs, route(costs, 1 if selector == "greedy" else 2)


def pack_cfg(states, timesteps, history_row=0, negative_row=1):
    """Candidate rows for CFG (wan_va_server.py:747-780): [all conditional,
    all unconditional] states and timesteps, and the history / context row
    of each ([row]*K + [negative_row]*K)."""
    k = states.shape[0]
    rows = torch.tensor([history_row] * k + [negative_row] * k, dtype=torch.int64, device=states.device)
    return torch.cat((states, states)), torch.cat((timesteps, timesteps)), rows


def cfg_combine(output, count, scale, out=None):
    """uncond + scale * (cond - uncond) over packed [cond | uncond] rows when
    scale > 1, else cond (wan_va_server.py:1936-1941)."""
    cond, uncond = output[:count], output[count:2 * count]
    if out is None:
        out = torch.empty_like(cond)
    _lib.check(_lib.load().wamb_cfg_combine(cond.data_ptr(), uncond.data_ptr(), _io(output), cond.numel(),
                                            float(scale), out.data_ptr(), _lib.stream_ptr()))
    return out


class NativeActionTarget:
    """Target directions of candidate action states from NativeWanModel in
    action mode, read-only over the KV history (update_cache=0 with
    candidate_cache_rows, model.py:624-660). states [K, L, A] time-major bf16
    (L = F H W positions), timesteps [K] fp32 -> [K, L, A] bf16. With
    guidance_scale > 1 the model's context must be prepared as [conditional,
    negative] and the KV history must hold the unconditional row at
    negative_row."""

    def __init__(self, native_model, action_grid, rotary_emb, history_row=0, guidance_scale=1.0,
                 negative_row=1):
        self.nm, self.grid, self.rope = native_model, tuple(action_grid), rotary_emb
        self.row, self.scale, self.neg = history_row, float(guidance_scale), negative_row
        self._rows = {}

    def __call__(self, states, timesteps):
        k = states.shape[0]
        F = self.grid[0]
        cfg = self.scale > 1.0
        if cfg:
            states, timesteps, rows = pack_cfg(states, timesteps, self.row, self.neg)
            ctx_rows = rows
        else:
            rows = self._rows.get(k)
            if rows is None:
                rows = self._rows[k] = torch.full((k,), self.row, dtype=torch.int64, device=states.device)
            ctx_rows = None
        n = states.shape[0]
        t = timesteps.reshape(n, 1).expand(n, F).contiguous()
        y = self.nm.forward({"action_tokens": states, "action_grid": self.grid, "timesteps": t,
                             "rotary_emb": self.rope}, 0, "pos", True, candidate_cache_rows=rows,
                            context_rows=ctx_rows)
        return cfg_combine(y, k, self.scale) if cfg else y


class GraphedTarget:
    """A target callable replayed from CUDA graphs, one per batch size,
    captured on first use over static input buffers: the loop's 1-row and
    7-row target forwards without per-call launch overhead. The returned
    tensor is the graph's static output (valid until the next call)."""

    def __init__(self, target):
        self.target = target
        self.graphs = {}

    def _capture(self, states, times):
        b = states.shape[0]
        st = states.clone()
        tt = times.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.target(st, tt)                  # warm-up: allocations, first-use setup
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = self.target(st, tt)
        self.graphs[b] = (g, st, tt, out)

    def __call__(self, states, times):
        b = states.shape[0]
        if b not in self.graphs:
            self._capture(states, times)
        g, st, tt, out = self.graphs[b]
        st.copy_(states)
        tt.copy_(times)
        g.replay()
        return out


class K2B2Speculative:
    """RealSpeculative.loop (real_speculative.py:32-109) on the device.

    target(states [b, 32, A], timesteps [b] fp32) -> directions [b, 32, A]
    (same dtype as the states); draft: a DraftPredictor; tau: the acceptance
    threshold. loop() returns the final [1, 32, A] state; self.rounds holds
    (step, depth, parent, child) per round (depth None for an ordinary target
    update)."""

    def __init__(self, target, draft, tau):
        if not (np.isfinite(tau) and tau >= 0):
            raise ValueError("tau must be finite and >= 0")
        self.target, self.draft, self.tau = target, draft, float(tau)
        self.rounds = []

    def loop(self, state, timesteps, deltas):
        n = len(timesteps)
        if len(deltas) != n or state.dim() != 3 or state.shape[0] != 1:
            raise ValueError("state [1, 32, A] and equal-length timesteps / deltas")
        dev, dt = state.device, state.dtype
        io = _io(state)
        A = state.shape[-1]
        N = 32 * A
        lib, st = _lib.load(), _lib.stream_ptr()
        tree = torch.empty(7, 32, A, dtype=dt, device=dev)        # root, parents, leaves
        tree[0].copy_(state[0])
        dirs = torch.empty(6, 32, A, dtype=dt, device=dev)        # dirs1[2], dirs2[2][2]
        prev = torch.empty(1, 32, A, dtype=dt, device=dev)
        scores = torch.empty(6, dtype=torch.float32, device=dev)
        rte = torch.empty(4, dtype=torch.int32, device=dev)
        ts = [float(t) for t in timesteps]
        ds = [float(d) for d in deltas]
        scal = torch.tensor([draft_scalars(ts[k], ds[k]) * 2 for k in range(n)], dtype=torch.float32,
                            device=dev).reshape(n, 2, 3)               # each row twice (two parents)
        times = torch.tensor(ts, dtype=torch.float32, device=dev)
        edges_d = (ctypes_int32 * 6)(0, 1, 2, 3, 4, 5)
        edges_t = (ctypes_int32 * 6)(0, 0, 1, 1, 2, 2)
        self.rounds = []
        i, have_prev = 0, False
        while i < n:
            if not have_prev or n - i < 3:
                v = self.target(tree[0:1], times[i:i + 1])
                _lib.check(lib.wamb_spec_expand(tree.data_ptr(), v.data_ptr(), io, 1, 1, N, ds[i], tree.data_ptr(),
                                                st))
                prev.copy_(v)
                have_prev = True
                self.rounds.append((i, None, None, None))
                i += 1
                continue
            self.draft.decode(tree[0:1], prev, scal[i, :1], out=dirs[0:2].view(1, 2, 32, A))
            _lib.check(lib.wamb_spec_expand(tree.data_ptr(), dirs.data_ptr(), io, 2, 2, N, ds[i],
                                            tree[1].data_ptr(), st))
            self.draft.decode(tree[1:3], dirs[0:2], scal[i + 1], out=dirs[2:6].view(2, 2, 32, A))
            _lib.check(lib.wamb_spec_expand(tree[1].data_ptr(), dirs[2].data_ptr(), io, 4, 2, N, ds[i + 1],
                                            tree[3].data_ptr(), st))
            tt = torch.cat((times[i:i + 1], times[i + 1:i + 2].expand(2), times[i + 2:i + 3].expand(4)))
            values = self.target(tree, tt).contiguous()
            sc = (ctypes_float * 6)(ds[i], ds[i], ds[i + 1], ds[i + 1], ds[i + 1], ds[i + 1])
            _lib.check(lib.wamb_spec_scores(dirs.data_ptr(), values.data_ptr(), io, N, 6, edges_d, edges_t, sc, 0,
                                            scores.data_ptr(), st))
            _lib.check(lib.wamb_spec_route(scores.data_ptr(), 0, self.tau, rte.data_ptr(), st))
            _lib.check(lib.wamb_spec_commit(rte.data_ptr(), values.data_ptr(), tree.data_ptr(), io, N, ds[i],
                                            ds[i + 1], ds[i + 2], tree.data_ptr(), prev.data_ptr(), st))
            depth, parent, child, _ = rte.tolist()
            self.rounds.append((i, depth, parent, child))
            i += depth + 1
        self.last_scores = scores
        return tree[0:1].clone()

