"""Golden fixtures that pin oracle/wan_model.py (the whole-model forward
around the blocks, and the flow-match scheduler) to the reference source.

Run in the build container, where the reference tree is mounted:
    python tests/golden/make_model_golden.py [REFERENCE_ROOT]
It AST-extracts WanTimeTextImageEmbedding and WanTransformer3DModel (with the
block classes) from the reference's
投机采样/wam-p0-worktree/wan_va/modules/model.py, supplies the diffusers
pieces it imports (not installed: ModelMixin / ConfigMixin become
nn.Module / object, and Timesteps, TimestepEmbedding,
PixArtAlphaTextProjection, FP32LayerNorm, FeedForward come from the oracle,
so those stay unpinned), loads wan_va/utils/scheduler.py as it is, runs
seeded fp32 CPU cases and writes tests/golden/model_cases.pt (inputs,
outputs, parameter checksums; weights are regenerated from the seed).

Nothing in the GPU tests, smoke() or bench.py runs this script.
"""
import ast
import math
import sys
from copy import deepcopy
from pathlib import Path

import torch
import torch.nn.functional as F
from einops import rearrange
from torch import nn

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from make_golden import MODEL_REL, UTILS_REL, _ff_factory, seeded_params  # noqa: E402
from oracle import wan_block as ob  # noqa: E402
from oracle import wan_model as om  # noqa: E402

SCHED_REL = "投机采样/wam-p0-worktree/wan_va/utils/scheduler.py"
NAMES = ("custom_sdpa", "WanRotaryPosEmbed", "WanAttention", "WanTransformerBlock",
         "WanTimeTextImageEmbedding", "WanTransformer3DModel")

# Small model: 2 heads (D 256), FFN 512, 2 layers, 4 latent channels,
# 30-d actions, 64-d text.
CFG = dict(patch_size=[1, 2, 2], num_attention_heads=2, attention_head_dim=128, in_channels=4,
           out_channels=4, action_dim=30, text_dim=64, freq_dim=256, ffn_dim=512, num_layers=2,
           cross_attn_norm=True, eps=1e-6)


def load_reference(root):
    src = (Path(root) / MODEL_REL).read_text()
    tree = ast.parse(src)
    body = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in NAMES]

    class FlexAttnFunc(nn.Module):
        pass

    ns = {"torch": torch, "nn": nn, "F": F, "math": math, "rearrange": rearrange, "deepcopy": deepcopy,
          "FP32LayerNorm": ob.FP32LayerNorm, "FeedForward": _ff_factory, "FlexAttnFunc": FlexAttnFunc,
          "flash_attn_func": None, "ModelMixin": nn.Module, "ConfigMixin": object,
          "register_to_config": lambda f: f, "Timesteps": om.Timesteps,
          "TimestepEmbedding": om.TimestepEmbedding,
          "PixArtAlphaTextProjection": lambda a, b, act_fn=None: om.PixArtAlphaTextProjection(a, b)}
    exec(compile(ast.Module(body=body, type_ignores=[]), str(Path(root) / MODEL_REL), "exec"), ns)
    utree = ast.parse((Path(root) / UTILS_REL).read_text())
    ubody = [n for n in utree.body if isinstance(n, ast.FunctionDef) and n.name == "get_mesh_id"]
    exec(compile(ast.Module(body=ubody, type_ignores=[]), UTILS_REL, "exec"), ns)
    sns = {}
    exec(compile((Path(root) / SCHED_REL).read_text(), SCHED_REL, "exec"), sns)
    return ns, sns


def model_inputs(ns, action_mode, seed):
    g = torch.Generator().manual_seed(seed)
    if action_mode:
        B, f, h, w = 2, 8, 4, 1
        x = torch.randn(B, CFG["action_dim"], f, h, w, generator=g)
        grid = ns["get_mesh_id"](f, h, w, 0, action=True)
        steps = torch.rand(B, f, generator=g) * 1000
    else:
        B, f, h, w = 1, 2, 8, 8
        x = torch.randn(B, CFG["in_channels"], f, h, w, generator=g)
        grid = ns["get_mesh_id"](f, h // 2, w // 2, 0)
        steps = torch.rand(B, f, generator=g) * 1000
    return {"noisy_latents": x, "text_emb": torch.randn(B, 16, CFG["text_dim"], generator=g),
            "grid_id": grid[None], "timesteps": steps}


def main(root):
    ns, sns = load_reference(root)
    torch.manual_seed(0)
    model = ns["WanTransformer3DModel"](**CFG, rope_max_seq_len=1024, pos_embed_seq_len=None,
                                        attn_mode="torch").eval()
    sums = seeded_params(model, seed=4242)
    cases = []
    for k, action_mode in enumerate((True, False)):
        inp = model_inputs(ns, action_mode, 8000 + k)
        with torch.no_grad():
            out = model(inp, update_cache=0, action_mode=action_mode)
        cases.append({"action_mode": action_mode, "inputs": inp, "out": out})
    sched = []
    for kw, n in (({"shift": 5.0, "sigma_min": 0.0, "extra_one_step": True}, 10), ({}, 50)):
        s = sns["FlowMatchScheduler"](**kw)
        s.set_timesteps(n)
        g = torch.Generator().manual_seed(n)
        sample, v = torch.randn(3, 7, generator=g), torch.randn(3, 7, generator=g)
        steps = [(float(t), s.step(v, t, sample)) for t in s.timesteps[:: max(1, n // 4)]]
        sched.append({"kwargs": kw, "n": n, "sigmas": s.sigmas.clone(), "timesteps": s.timesteps.clone(),
                      "sample": sample, "v": v, "steps": steps})
    fixtures = {"model_source": MODEL_REL, "scheduler_source": SCHED_REL, "config": CFG, "seed": 4242,
                "param_sums": sums, "cases": cases, "scheduler": sched}
    out = HERE / "model_cases.pt"
    torch.save(fixtures, out)
    print(f"wrote {out} ({out.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
