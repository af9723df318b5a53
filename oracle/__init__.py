"""CPU oracle for the Wan-DiT block hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
(`--impl reference` and the `cpu_baseline` object) may import this package,
and only as the checker or as the timed CPU reference. The product path
(wam-egale_b200/) never imports it and has no CPU fallback.

Contents:
  wan_block.py   plain PyTorch (fp32, CPU) restatement of the reference's
                 WanTransformerBlock / WanAttention / "original" KV cache /
                 WanRotaryPosEmbed / get_mesh_id, each citing the reference
                 file:line it follows.
  wan_model.py   the whole-model inference forward around the blocks
                 (embedders, output norm and projection) and the flow-match
                 scheduler (model.py:203-240, 797-872, 1028-1116;
                 scheduler.py:6-89).
  fp8.py         the FP8-E4M3 GEMM path (no reference counterpart): row
                 quantization and a block copy with quantized GEMMs.
  speculative.py speculative action decoding around the target model: the
                 FastWAM draft predictor, weighted-L2 edge scores, the K2/B2
                 and K3/B2 route rules and the K2/B2 loop
                 (fastwam-base/fullcode-v1/draft.py, real_speculative.py;
                 wam-p0-worktree/wan_va/utils/p0_k3_b2.py), pinned by
                 tests/golden/make_spec_golden.py.

Parity pin: tests/golden/make_golden.py runs the reference's own model.py
source (AST-extracted, in the build container where the reference is
mounted) on seeded inputs and commits the outputs as fixtures;
tests/test_oracle_golden.py checks this restatement against them.
The diffusers pieces the reference imports (FP32LayerNorm, FeedForward,
Timesteps/TimestepEmbedding) are not in the reference tree; the first two are
restated from the reference's own native restatements (pinned indirectly),
the timestep embedder is outside the block and unpinned.
"""
