"""Generate the golden fixtures that pin the oracle to the reference source.

Run in the build container, where the reference tree is mounted:
    python tests/golden/make_golden.py [REFERENCE_ROOT]
It AST-extracts `custom_sdpa`, `WanRotaryPosEmbed`, `WanAttention` and
`WanTransformerBlock` from the reference's
投机采样/wam-p0-worktree/wan_va/modules/model.py (the method the reference
itself uses for its CPU contract tests), supplies the two diffusers modules
it imports (FP32LayerNorm, FeedForward; diffusers is not installed) from
oracle/wan_block.py, runs seeded fp32 CPU cases through the reference code
and writes tests/golden/block_cases.pt: the inputs, the outputs and the KV
cache state after every call. Weights are not stored: they are regenerated
from the seed and checked against stored checksums.

Nothing in the GPU tests, smoke() or bench.py runs this script.
"""
import ast
import sys
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn
from einops import rearrange

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import wan_block as ob  # noqa: E402

MODEL_REL = "投机采样/wam-p0-worktree/wan_va/modules/model.py"
UTILS_REL = "投机采样/wam-p0-worktree/wan_va/utils/utils.py"
NAMES = ("custom_sdpa", "WanRotaryPosEmbed", "WanAttention", "WanTransformerBlock")


def load_reference(root):
    src = (Path(root) / MODEL_REL).read_text()
    tree = ast.parse(src)
    body = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in NAMES]
    module = ast.Module(body=body, type_ignores=[])

    class FlexAttnFunc(nn.Module):  # only referenced by isinstance checks
        pass

    ns = {"torch": torch, "nn": nn, "F": F, "math": __import__("math"), "rearrange": rearrange,
          "FP32LayerNorm": ob.FP32LayerNorm, "FeedForward": _ff_factory,
          "FlexAttnFunc": FlexAttnFunc, "flash_attn_func": None}
    exec(compile(module, str(Path(root) / MODEL_REL), "exec"), ns)
    usrc = (Path(root) / UTILS_REL).read_text()
    utree = ast.parse(usrc)
    ubody = [n for n in utree.body if isinstance(n, ast.FunctionDef) and n.name == "get_mesh_id"]
    exec(compile(ast.Module(body=ubody, type_ignores=[]), UTILS_REL, "exec"), ns)
    return ns


def _ff_factory(dim, inner_dim=None, activation_fn=None):
    assert activation_fn == "gelu-approximate"
    return ob.FeedForward(dim, inner_dim)


def seeded_params(block, seed):
    """Deterministic weights; returns checksums (sum, sum of squares) per tensor."""
    g = torch.Generator().manual_seed(seed)
    sums = {}
    with torch.no_grad():
        for name, p in sorted(block.named_parameters()):
            t = torch.randn(p.shape, generator=g)
            if name.endswith("scale_shift_table"):
                t = t / p.shape[-1] ** 0.5
            elif "norm" in name and name.endswith("weight"):
                t = 1.0 + 0.1 * t
            elif "norm" in name and name.endswith("bias"):
                t = 0.1 * t
            else:
                t = 0.02 * t
            p.copy_(t)
            sums[name] = (float(t.double().sum()), float(t.double().square().sum()))
    return sums


def case_inputs(B, Q, D, C, seed, temb_len, rope_ns):
    # Inputs are bf16-representable so that they are stored exactly as bf16.
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, Q, D, generator=g).bfloat16().float()
    ctx = torch.randn(B, C, D, generator=g).bfloat16().float()
    temb = (0.5 * torch.randn(B, temb_len, 6, D, generator=g)).bfloat16().float()
    grid = rope_ns["get_mesh_id"](max(1, Q // 8), 4, 2, 0)[:, :Q]
    if grid.shape[1] < Q:
        grid = torch.cat([grid, rope_ns["get_mesh_id"](1, Q - grid.shape[1], 1, 0, action=True)], 1)
    rope = rope_ns["WanRotaryPosEmbed"](128, [1, 2, 2], 1024)(grid[None])[:, :, None]
    return x, ctx, temb, rope


# (name, dim, ffn, heads, pool or None, calls[(B, Q, C, temb_len, update, candidate_rows)])
CASES = [
    ("no_cache", 256, 512, 2, None, [(2, 40, 24, 1, 0, None)]),
    ("per_token_temb", 256, 512, 2, None, [(1, 33, 17, 33, 0, None)]),
    # Evictions here always free whole chunks (all slots of the smallest id):
    # the reference's CPU argsort is not stable, so an eviction that splits a
    # chunk picks implementation-defined slots and cannot serve as a pin.
    ("kv_lifecycle", 256, 512, 2, 120,
     [(2, 40, 24, 1, 2, None), (2, 40, 24, 1, 2, None), (2, 40, 24, 1, 0, None),
      (2, 40, 24, 1, 1, None), (2, 40, 24, 1, 0, None), (2, 40, 24, 1, 2, None),
      (2, 40, 24, 1, 1, None)]),
    ("candidates", 256, 512, 2, 200,
     [(2, 70, 24, 1, 2, None), (2, 70, 24, 1, 2, None), (4, 16, 24, 16, 0, [0, 1, 1, 0])]),
]


def main(root):
    ref = load_reference(root)
    fixtures = {"model_source": MODEL_REL, "cases": []}
    for ci, (name, D, Fd, H, pool, calls) in enumerate(CASES):
        torch.manual_seed(0)
        blk = ref["WanTransformerBlock"](D, Fd, H, cross_attn_norm=True, eps=1e-6, attn_mode="torch")
        sums = seeded_params(blk, seed=1000 + ci)
        blk.eval()
        if pool is not None:
            blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, calls[0][0])
        recs = []
        for k, (B, Q, C, tl, update, rows) in enumerate(calls):
            x, ctx, temb, rope = case_inputs(B, Q, D, C, 7000 + 10 * ci + k, tl, ref)
            kw = {"update_cache": update}
            if rows is not None:
                kw["candidate_cache_rows"] = torch.tensor(rows, dtype=torch.int64)
            with torch.no_grad():
                out = blk(x, ctx, temb, rope, **kw)
            rec = {"x": x.bfloat16(), "ctx": ctx.bfloat16(), "temb": temb.bfloat16(), "rope": rope,
                   "update": update, "rows": rows, "out": out}
            if pool is not None:
                c = blk.attn1.attn_caches["pos"]
                rec["cache"] = {"id": c["id"].clone(), "mask": c["mask"].clone(),
                                "is_pred": c["is_pred"].clone()}
                if k == len(calls) - 1:  # pool rows only after the last call (fixture size)
                    seen = (c["id"] >= 0).nonzero().squeeze(-1)
                    rec["cache"]["slots"] = seen
                    rec["cache"]["k"] = c["k"][:, seen].clone()
                    rec["cache"]["v"] = c["v"][:, seen].clone()
            recs.append(rec)
        fixtures["cases"].append({"name": name, "dim": D, "ffn": Fd, "heads": H, "pool": pool,
                                  "seed": 1000 + ci, "param_sums": sums, "calls": recs})
    out = HERE / "block_cases.pt"
    torch.save(fixtures, out)
    print(f"wrote {out} ({out.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
