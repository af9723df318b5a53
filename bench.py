"""Benchmark: 30-layer 5B-shape Wan-DiT denoise step on B200 (one process per GPU).

Workload (BASELINE configs[4] per-GPU slice, configs[2] per rollout): every
rank holds 8 independent rollouts, each one 880-token chunk (848 video + 32
action tokens) attending to its own 3520-token self-KV history plus itself,
with a prepared 512-token cross-K/V, through 30 layers of D 3072 / 24x128
heads / FFN 14336, bf16 tensor-core math, update_cache=0 (the pool mask is
restored, so every step sees the same cache). A "step" is one 30-layer
denoise step of all 8 rollouts; weights (9.8 GB) and KV pools (13 GB) are far
larger than L2, so no flush is needed between steps. Under torchrun each
rank runs its own 8 rollouts (weak scaling) and the 32 action-token outputs
of every rollout are all-gathered over NCCL after each step.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Rank 0 prints one JSON line (see the keys below). `value` is chunk-steps/s
for the whole job (rollouts x ranks / step time), `ms_per_step` is the DiT
denoise-step time. `--impl reference` times the reference algorithm's CPU
implementation (the fp32 oracle port) on the host cores instead.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "wam-egale_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "chunk_denoise_steps_per_s"
UNIT = "chunk-steps/s"
CHUNK_STEPS = 10  # FastWAM denoise updates per action chunk (real_speculative.py:33,107)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) of one FFN1 + GELU launch at the bench shape
# (M 7040, N 14336, K 3072, bf16), from one ncu capture of the same kernel:
# 212.1 MB read + 186.6 MB written (algorithmic: 333.3 MB).
FFN1_TRAFFIC_BYTES = 398.7e6


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def workload_config(n_gpus, batch):
    return {"workload": "cfg4 slice: 8 rollouts/GPU of cfg2 (30-layer 5B-shape Wan-DiT denoise step, "
                        "880-token chunk = 848 video + 32 action, 3520-token self-KV history, "
                        "512-token prepared cross-K/V)",
            "model": "Wan-DiT block stack D3072 H24x128 F14336 L30",
            "global_batch": batch * n_gpus, "seq_len": 880, "kv_history": 3520, "context": 512,
            "parallelism": f"rollouts sharded, {batch}/GPU" + (", NCCL all_gather of action outputs"
                                                                if n_gpus > 1 else ""),
            "l2": "inputs larger than L2 (9.8 GB weights + 13 GB KV per step)",
            "chunk_steps_per_action_chunk": CHUNK_STEPS}


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(",") for r in Path(self.path).read_text().splitlines() if r.strip()]
        os.unlink(self.path)
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                mhz.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not mhz:
            return None
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# --------------------------------------------------------------- CPU side
class CpuReference:
    """The reference algorithm on the host cores: the fp32 oracle restatement
    of the block (oracle/wan_block.py) for ONE cfg2 rollout (880 tokens
    attending to a 3520-token history + itself, 512 context tokens). A step
    is a whole 30-layer denoise step of that rollout: the hidden states pass
    through 30 block forwards (update_cache=0). One block's weights serve all
    30 layers (same FLOPs and bytes per layer as 30 distinct blocks, without
    11.7 GB of fp32 host weights)."""

    def __init__(self):
        from oracle import wan_block as ob
        from wam_ops import configs

        torch.set_num_threads(os.cpu_count() or 1)
        cfg = self.cfg = configs.PRESETS["cfg2"]
        D, H, F, Q = cfg.dim, cfg.heads, cfg.ffn, cfg.tokens
        g = torch.Generator().manual_seed(0)
        blk = ob.WanTransformerBlock(D, F, H, cross_attn_norm=True, eps=1e-6).eval()
        with torch.no_grad():
            for name, p in blk.named_parameters():
                if name.endswith("weight") and "norm" not in name:
                    p.copy_(torch.randn(p.shape, generator=g) * 0.02)
        pool, hist = cfg.pool_chunks * Q, cfg.history_chunks * Q
        blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, 1)
        c = blk.attn1.attn_caches["pos"]
        c["k"].normal_(generator=g)
        c["v"].normal_(generator=g)
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist) // Q
        self.blk = blk
        self.args = (torch.randn(1, Q, D, generator=g), torch.randn(1, cfg.context, D, generator=g),
                     configs.make_temb(cfg, 1, "cpu", g), configs.chunk_rope(cfg))

    def step(self, layers=None):
        """Seconds for `layers` (default all 30) chained block forwards."""
        x, ctx, temb, rope = self.args
        with torch.no_grad():
            t0 = time.perf_counter()
            for _ in range(self.cfg.layers if layers is None else layers):
                x = self.blk(x, ctx, temb, rope, update_cache=0)
            return time.perf_counter() - t0

    def describe(self):
        return (f"one 30-layer denoise step of one cfg2 rollout per sample (880 tokens, 4400 visible "
                f"keys, 512 context, fp32, {self.cfg.layers} chained block forwards)")


PER_ROLLOUT = ("per-rollout throughput: rollouts are independent and the CPU reference's cost is "
               "linear in them, so chunk-steps/s of one rollout per step is the comparable unit")


def cpu_reference_rate(samples=2):
    """(chunk-steps/s, threads, seconds per step, sample text) of the CPU
    reference: `samples` whole 30-layer steps after a one-layer warm-up."""
    ref = CpuReference()
    ref.step(1)
    dt = sum(ref.step() for _ in range(samples)) / samples
    return 1.0 / dt, torch.get_num_threads(), dt, ref.describe() + f"; {samples} samples"


def run_reference(args):
    """--impl reference: the reference's CPU path on the host (rank 0 only);
    each timed step is a whole 30-layer step of one rollout, each warm-up
    step one layer forward."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n = args.gpus
    ref = CpuReference()
    for _ in range(args.warmup):
        ref.step(1)
    t0 = time.perf_counter()
    per_step = [ref.step() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    step_s = sum(per_step) / len(per_step)
    value = 1.0 / step_s
    sample = ref.describe()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * step_s,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, cfg2 shapes)",
            "config": workload_config(n, 1) | {"sample_per_step": sample, "unit_note": PER_ROLLOUT,
                                               "warmup_step": "one layer forward"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": wall}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- GPU side
def time_graph(run, steps, stream):
    """ms per call of `run` over `steps` calls, CUDA events on `stream`."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def step_roofline(cfg, batch, ms, fp8=False):
    """Algorithmic FLOPs of one step of `batch` rollouts against the measured
    sustained bf16 peak (the E4M3 GEMMs at twice that rate in fp8 mode)."""
    pk, pk_kind = peaks()
    gemm_flops, attn_flops = stack_flops(cfg, split=True)
    sus = pk["bf16_tflops_sustained"] * 1e12
    tc = 2.0 if fp8 else 1.0
    floor_s = batch * (gemm_flops / (sus * tc) + attn_flops / sus)
    flops = (gemm_flops + attn_flops) * batch
    return {"achieved": flops / (ms / 1000.0) / 1e12, "unit": "TFLOP/s",
            "peak": pk["bf16_tflops_sustained"] * tc, "frac": floor_s / (ms / 1000.0),
            "peak_source": f"{pk_kind} bf16 sustained" + (
                "; frac = (GEMM FLOPs at 2x + attention FLOPs at 1x) / time" if fp8 else ""),
            "algorithmic_flops_per_step": flops}


class ActionGather:
    """NCCL all_gather of every rollout's action rows after each step, off the
    compute stream: the step's last kernel copies the rows into a two-slot
    ring on the compute stream, a side stream runs the collective, and the
    compute stream waits only before it rewrites a ring slot whose gather
    (two steps back) may still be reading it. Ranks therefore do not step in
    lockstep with the slowest one; `drain()` joins the side stream back."""

    def __init__(self, out, action_tokens, world):
        B, _, D = out.shape
        self.out, self.A = out, action_tokens
        self.src = [torch.empty(B, action_tokens, D, dtype=out.dtype, device=out.device) for _ in range(2)]
        self.dst = [torch.empty(world * B, action_tokens, D, dtype=out.dtype, device=out.device)
                    for _ in range(2)]
        self.side = torch.cuda.Stream(device=out.device)
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.gathered = [None, None]
        self.k = 0

    def __call__(self):
        import torch.distributed as dist
        i = self.k % 2
        cur = torch.cuda.current_stream()
        if self.gathered[i] is not None:
            cur.wait_event(self.gathered[i])
        self.src[i].copy_(self.out[:, -self.A:])
        self.copied[i].record(cur)
        self.side.wait_event(self.copied[i])
        with torch.cuda.stream(self.side):
            dist.all_gather_into_tensor(self.dst[i], self.src[i])
            ev = torch.cuda.Event()
            ev.record(self.side)
        self.gathered[i] = ev
        self.k += 1

    def drain(self):
        torch.cuda.current_stream().wait_stream(self.side)


class PipelinedIO:
    """Host <-> device copies of a graph-replayed step overlapped with the
    steps around it, as a serving loop runs them. A copy stream brings step
    k+1's inputs from pinned host memory into one of two device staging sets
    and returns step k-1's output from one of two staging buffers while step
    k computes; the compute stream moves staging -> the graph's static
    inputs and its static output -> staging with device copies around each
    replay. Every step still copies its own inputs in and its output out."""

    def __init__(self, inputs, out, host_out):
        # inputs: [(static device tensor, pinned host tensor)]; out: static output
        dev = out.device
        self.inputs, self.out, self.host_out = inputs, out, host_out
        self.stage_in = [[torch.empty_like(d) for d, _ in inputs] for _ in range(2)]
        self.stage_out = [torch.empty_like(out) for _ in range(2)]
        self.cs = torch.cuda.Stream(device=dev)
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.in_free = [torch.cuda.Event() for _ in range(2)]
        self.out_ready = [torch.cuda.Event() for _ in range(2)]
        self.out_free = [torch.cuda.Event() for _ in range(2)]

    def _h2d(self, b, first):
        with torch.cuda.stream(self.cs):
            if not first:
                self.cs.wait_event(self.in_free[b])
            for st, (_, h) in zip(self.stage_in[b], self.inputs):
                st.copy_(h, non_blocking=True)
            self.in_ready[b].record(self.cs)

    def run(self, steps, step):
        cur = torch.cuda.current_stream()
        self.cs.wait_stream(cur)
        self._h2d(0, True)
        for k in range(steps):
            b = k % 2
            cur.wait_event(self.in_ready[b])
            for (d, _), st in zip(self.inputs, self.stage_in[b]):
                d.copy_(st)
            self.in_free[b].record(cur)
            if k + 1 < steps:
                self._h2d(1 - b, k == 0)
            step()
            if k >= 2:
                cur.wait_event(self.out_free[b])
            self.stage_out[b].copy_(self.out)
            self.out_ready[b].record(cur)
            with torch.cuda.stream(self.cs):
                self.cs.wait_event(self.out_ready[b])
                self.host_out.copy_(self.stage_out[b], non_blocking=True)
                self.out_free[b].record(self.cs)
        cur.wait_stream(self.cs)


def run_stack_config(name, dev, steps, warmup, fp8=False, seed=0):
    """One graph-replayed 30-layer step of a 1-GPU config: cfg2 (batch 1,
    880-token chunk over its 3520-token history) or cfg1 (batch 1, 1592
    tokens of the D 1536 stack, no self-KV history); prepared cross K/V."""
    from wam_ops import _lib, configs
    from wam_ops.stack import NativeStack

    cfg = configs.PRESETS[name]
    B, Q, D = cfg.batch, cfg.tokens, cfg.dim
    gen = torch.Generator(device=dev).manual_seed(seed)
    blocks = configs.build_blocks(cfg, dev, seed=seed)
    if cfg.history_chunks:
        configs.fill_history(blocks, cfg, dev, gen, pool_batch=B)
    stack = NativeStack(blocks, fp8=fp8)
    ctx = torch.randn(B, cfg.context, D, generator=gen, device=dev).bfloat16()
    stack.prepare_context(ctx)
    x = torch.randn(B, Q, D, generator=gen, device=dev).bfloat16()
    temb = configs.make_temb(cfg, B, dev, gen)
    rope = configs.chunk_rope(cfg, f_shift=cfg.history_chunks).to(dev)
    stack.capture(x, ctx, temb, rope, warmup=1)
    stream = torch.cuda.current_stream()
    clocks = Clocks(dev.index)
    clocks.start()
    time.sleep(0.3)          # the sampler starts; the warm-up then brings the clocks back up
    for _ in range(warmup):
        stack.replay()
    ms = time_graph(stack.replay, steps, stream)
    clk = clocks.stop()
    code = _lib.device_status()
    hist = cfg.history_chunks * Q
    line = {"workload": f"{name}: 30-layer Wan-DiT denoise step, D{D} H{cfg.heads}x128 F{cfg.ffn}, batch {B}, "
                        f"{Q} tokens" + (f" over a {hist}-token self-KV history" if hist else "")
                        + f", {cfg.context}-token prepared cross-K/V",
            "dtype": "fp8-e4m3 GEMMs, bf16 attention" if fp8 else "bf16",
            "ms_per_step": ms, "steps_per_s": 1000.0 / ms,
            "step_roofline": step_roofline(cfg, B, ms, fp8),
            "gpu_launches": stack.launches_per_step(with_cache=bool(hist)) * steps,
            "clocks": clk, "device_error": code}
    del stack, blocks
    torch.cuda.empty_cache()
    return line


def run_native(args):
    from wam_ops import _lib, configs, ops
    from wam_ops.stack import NativeStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    cfg = configs.PRESETS["cfg4"]
    B, Q, D = cfg.batch, cfg.tokens, cfg.dim
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    torch.set_grad_enabled(False)

    blocks = configs.build_blocks(cfg, dev, seed=1234)
    configs.fill_history(blocks, cfg, dev, gen, pool_batch=B)
    ctx = torch.randn(B, cfg.context, D, generator=gen, device=dev).bfloat16()
    x = torch.randn(B, Q, D, generator=gen, device=dev).bfloat16()
    temb = configs.make_temb(cfg, B, dev, gen)
    rope = configs.chunk_rope(cfg).to(dev)
    A = 32  # action tokens per rollout
    stream = torch.cuda.current_stream()

    def measure(fp8):
        """(ms per step, clocks, stack, static buffers, step function)."""
        stack = NativeStack(blocks, fp8=fp8)
        stack.prepare_context(ctx)
        torch.cuda.synchronize()
        if _lib.device_status() != 0:
            raise RuntimeError("device error during setup")
        static = stack.capture(x, ctx, temb, rope, warmup=1)
        gather = ActionGather(static["out"], A, world) if pg is not None else None

        def step():
            out = stack.replay()
            if gather is not None:
                gather()
            return out

        clocks = Clocks(local)
        clocks.start()
        time.sleep(0.3)      # the sampler starts; the warm-up then brings the clocks back up
        for _ in range(args.warmup):
            step()
        if gather is not None:
            gather.drain()
        torch.cuda.synchronize()
        if _lib.device_status() != 0:
            raise RuntimeError("device error during warm-up")
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

        def timed():
            for _ in range(args.steps):
                step()
            if gather is not None:
                gather.drain()
        ms = time_graph(timed, 1, stream) / args.steps
        clk = clocks.stop()
        if pg is not None:
            pg.barrier()
        t = torch.tensor([ms], device=dev)
        if pg is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return t.item(), clk, stack, static, step, gather

    ms, clk, stack, static, step, gather = measure(False)
    value = B * world / (ms / 1000.0)
    dev_code = _lib.device_status()

    # ---- e2e through the public API: pinned host input -> step -> host output
    hx = x.cpu().pin_memory()
    ht = temb.cpu().pin_memory()
    hout = torch.empty(B, Q, D, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        stack.replay(hx.to(dev, non_blocking=True), ht.to(dev, non_blocking=True))
        hout.copy_(static["out"], non_blocking=True)
    if gather is not None:
        gather.drain()
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()

    def e2e_serial():
        for _ in range(args.steps):
            static["x"].copy_(hx, non_blocking=True)
            static["temb"].copy_(ht, non_blocking=True)
            step()
            hout.copy_(static["out"], non_blocking=True)
        if gather is not None:
            gather.drain()
    pio = PipelinedIO([(static["x"], hx), (static["temb"], ht)], static["out"], hout)

    def e2e_pipelined():
        pio.run(args.steps, step)
        if gather is not None:
            gather.drain()
    e2e_pipelined()   # warm the copy stream and staging buffers
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    ms_serial = time_graph(e2e_serial, 1, stream) / args.steps
    if pg is not None:
        pg.barrier()
    ms_e2e = time_graph(e2e_pipelined, 1, stream) / args.steps
    t = torch.tensor([ms_e2e, ms_serial], device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_e2e, ms_serial = t.tolist()
    e2e = {"value": B * world / (ms_e2e / 1000.0), "unit": UNIT,
           "h2d_bytes_per_step": hx.numel() * 2 + ht.numel() * 4,
           "d2h_bytes_per_step": hout.numel() * 2, "ms_per_step": ms_e2e,
           "copies": "each step's input copied in from pinned host memory and its output copied out, on a "
                     "copy stream overlapped with the neighbouring steps (PipelinedIO)",
           "serial_ms_per_step": ms_serial}
    launches = stack.launches_per_step(with_cache=True) * args.steps
    del stack, static, step, gather
    torch.cuda.empty_cache()

    if args.step_only:   # ncu launch lists of the step: skip the sub-runs
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                              "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                              "note": "--step-only: no fp8 / configs / cpu sub-runs"}), flush=True)
        if pg is not None:
            pg.barrier()
            pg.destroy_process_group()
        return 0
    # ---- the same workload with E4M3 GEMMs (configs[4]'s second run)
    ms8, clk8, stack8, static8, step8, gather8 = measure(True)
    fp8 = {"value": B * world / (ms8 / 1000.0), "unit": UNIT, "ms_per_step": ms8,
           "dtype": "fp8-e4m3 GEMMs (per-channel weight / per-token activation scales), bf16 attention",
           "step_roofline": step_roofline(cfg, B, ms8, fp8=True),
           "gpu_launches": stack8.launches_per_step(with_cache=True) * args.steps, "clocks": clk8}
    w8_first = stack8.layers[0].native.w8[23], stack8.layers[0].native.w8_scale[23]
    del stack8, static8, step8, gather8

    # ---- roofline of the dominant kernel (FFN1 GEMM + GELU, M = 8 x 880)
    M, F = B * Q, cfg.ffn
    blk0 = blocks[0]
    a = torch.randn(M, D, generator=gen, device=dev).bfloat16()
    w1, b1 = blk0.ffn.net[0].proj.weight, blk0.ffn.net[0].proj.bias
    act = torch.empty(M, F, dtype=torch.bfloat16, device=dev)
    pk, pk_kind = peaks()
    flops = 2.0 * M * F * D

    def kernel_rate(run):
        for _ in range(3):
            run()
        return time_graph(run, 20, stream)
    k_ms = kernel_rate(lambda: ops.linear(a, w1, b1, epilogue=_lib.EPI_GELU, out=act))
    achieved = flops / (k_ms / 1000.0) / 1e12
    kpeak = pk["bf16_tflops"]
    roof = {"kernel": "gemm_tc2_kernel<bf16> (2-CTA 256x256 tiles) FFN1+GELU (M 7040, N 14336, K 3072)",
            "bound": "tensor", "achieved": achieved, "peak": kpeak, "unit": "TFLOP/s",
            "frac": achieved / kpeak, "traffic": FFN1_TRAFFIC_BYTES,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of "
                              "`bench.py --workload kernel --case ffn1 --m 7040` (same kernel and shape)",
            "peak_source": f"{pk_kind} bf16 burst", "ms_per_launch": k_ms,
            "algorithmic_flops_per_launch": flops}
    a8, sa = ops.quantize_rows(a)
    k8_ms = kernel_rate(lambda: ops.linear(a8, w8_first[0], b1, epilogue=_lib.EPI_GELU, out=act, a_scale=sa,
                                           w_scales=w8_first[1]))
    # No fp8 GEMM peak is measured on this pool: the E4M3 tensor rate is
    # twice the bf16 one on B200, so its denominator is 2x the bf16 burst.
    fp8["roofline"] = {"kernel": "gemm_tc2_kernel<E4M3> FFN1+GELU (M 7040, N 14336, K 3072)", "bound": "tensor",
                       "achieved": flops / (k8_ms / 1000.0) / 1e12, "peak": 2 * kpeak, "unit": "TFLOP/s",
                       "frac": flops / (k8_ms / 1000.0) / 1e12 / (2 * kpeak),
                       "peak_source": f"{pk_kind} bf16 burst x 2 for E4M3", "ms_per_launch": k8_ms}
    del w8_first, a8, sa, act, a

    line = None
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded weights N(0,0.02), "
                "zero biases, N(0,1) hidden/context, random unit-scale KV history)",
                "config": workload_config(world, B) | {"action_chunks_per_s": value / CHUNK_STEPS},
                "roofline": roof, "step_roofline": step_roofline(cfg, B, ms), "e2e": e2e,
                "fp8": fp8, "gpu_launches": launches, "clocks": clk, "device_error": dev_code}
    del blocks
    torch.cuda.empty_cache()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        if world == 1:
            # The configs the north-star target is quoted on, timed on the same GPU.
            line["configs"] = {n: run_stack_config(n, dev, args.steps, args.warmup, seed=7 + i)
                               for i, n in enumerate(("cfg2", "cfg1"))}
            # cfg2 with the E4M3 GEMMs (configs[4]'s second run, at batch 1).
            line["configs"]["cfg2_fp8"] = run_stack_config("cfg2", dev, args.steps, args.warmup, fp8=True,
                                                           seed=7)
        if world == 1 and not args.no_cpu_baseline:
            v, th, dt, sample = cpu_reference_rate()
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": th, "kind": "port",
                                    "sample": sample, "unit_note": PER_ROLLOUT}
        print(json.dumps(line), flush=True)
    return 0


def run_config(args):
    """--workload cfg2 / cfg1: the 1-GPU config's step as its own line."""
    from wam_ops import configs

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    torch.set_grad_enabled(False)
    r = run_stack_config(args.workload, dev, args.steps, args.warmup, fp8=args.fp8, seed=7)
    cfg = configs.PRESETS[args.workload]
    line = {"metric": "denoise_steps_per_s", "value": r["steps_per_s"], "unit": "denoise-steps/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": r["dtype"],
            "data": "synthetic (seeded weights N(0,0.02), zero biases, N(0,1) hidden/context"
                    + (", random unit-scale KV history)" if cfg.history_chunks else ")"),
            "config": {"workload": r["workload"], "global_batch": cfg.batch, "seq_len": cfg.tokens,
                       "kv_history": cfg.history_chunks * cfg.tokens, "context": cfg.context,
                       "l2": "inputs larger than L2 (weights streamed every step)"},
            "step_roofline": r["step_roofline"], "roofline": dict(r["step_roofline"], bound="tensor",
                                                                  kernel="whole step"),
            "gpu_launches": r["gpu_launches"], "clocks": r["clocks"], "device_error": r["device_error"]}
    print(json.dumps(line), flush=True)
    return 0


def run_verify(args):
    """--workload cfg3: one 30-layer speculative-verify step: 4 candidate
    chunks x 32 action tokens attending to a read-only 3520-token history
    (candidate_cache_rows = 0 for every candidate) plus their own K/V, 512
    prepared context tokens, per-token temb. HBM-bound (weight streaming):
    the roofline line is bytes / time against the measured copy bandwidth.
    Under torchrun the candidates are split over the ranks (2 + 2 on 2
    GPUs): rank 0's KV history is NCCL-broadcast once into every rank's own
    memory before timing, each rank verifies its candidates, and their
    outputs are all-gathered after every step on a side stream."""
    from wam_ops import _lib, configs
    from wam_ops.rollouts import broadcast_cache, shard
    from wam_ops.stack import NativeStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    cfg = configs.PRESETS["cfg3"]
    B_all, Q, D, F = cfg.candidates, cfg.tokens, cfg.dim, cfg.ffn
    mine = list(shard(B_all, world, rank))
    B = len(mine)
    gen = torch.Generator(device=dev).manual_seed(4321)
    torch.set_grad_enabled(False)
    blocks = configs.build_blocks(cfg, dev, seed=4321)
    configs.fill_history(blocks, cfg, dev, gen, pool_batch=1)
    bcast = None
    if pg is not None:
        torch.cuda.synchronize()
        pg.barrier()
        t0 = time.perf_counter()
        nbytes = broadcast_cache(blocks, src=0)
        torch.cuda.synchronize()
        bcast = {"bytes_per_rank": nbytes, "ms": 1000.0 * (time.perf_counter() - t0)}
    stack = NativeStack(blocks, fp8=args.fp8)
    ctx = torch.randn(1, cfg.context, D, generator=gen, device=dev).bfloat16()
    stack.prepare_context(ctx)
    x_all = torch.randn(B_all, Q, D, generator=gen, device=dev).bfloat16()
    temb_all = configs.make_temb(cfg, B_all, dev, gen, per_token=Q)
    x, temb = x_all[mine].contiguous(), temb_all[mine].contiguous()
    rope = configs.chunk_rope(cfg, f_shift=cfg.history_chunks).to(dev)
    rows = torch.zeros(B, dtype=torch.int64, device=dev)
    static = stack.capture(x, ctx, temb, rope, candidate_cache_rows=rows, warmup=1)
    gather = ActionGather(static["out"], Q, world) if pg is not None else None

    def step():
        stack.replay()
        if gather is not None:
            gather()

    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)          # the sampler starts; the warm-up then brings the clocks back up
    for _ in range(args.warmup):
        step()
    if gather is not None:
        gather.drain()
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError("device error during warm-up")
    stream = torch.cuda.current_stream()
    if pg is not None:
        pg.barrier()

    def timed():
        for _ in range(args.steps):
            step()
        if gather is not None:
            gather.drain()
    ms = time_graph(timed, 1, stream) / args.steps
    clk = clocks.stop()
    hx, ht = x.cpu().pin_memory(), temb.cpu().pin_memory()
    hout = torch.empty(B, Q, D, dtype=torch.bfloat16).pin_memory()

    def e2e_serial():
        for _ in range(args.steps):
            static["x"].copy_(hx, non_blocking=True)
            static["temb"].copy_(ht, non_blocking=True)
            step()
            hout.copy_(static["out"], non_blocking=True)
        if gather is not None:
            gather.drain()
    pio = PipelinedIO([(static["x"], hx), (static["temb"], ht)], static["out"], hout)

    def e2e_pipelined():
        pio.run(args.steps, step)
        if gather is not None:
            gather.drain()
    e2e_pipelined()   # warm the copy stream and staging buffers
    torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    ms_serial = time_graph(e2e_serial, 1, stream) / args.steps
    if pg is not None:
        pg.barrier()
    ms_e2e = time_graph(e2e_pipelined, 1, stream) / args.steps
    if pg is not None:
        t = torch.tensor([ms, ms_e2e, ms_serial], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, ms_e2e, ms_serial = t.tolist()
    dev_code = _lib.device_status()
    # Algorithmic bytes of one step on one GPU: every GEMM weight once (self
    # q/k/v/out, cross q/out, FFN), the visible history K/V once, the
    # prepared cross K/V (each GPU streams all of them for its candidates).
    wbytes = 1 if args.fp8 else 2
    hist = cfg.history_chunks * configs.PRESETS["cfg2"].tokens
    per_layer = (6 * D * D + 2 * D * F) * wbytes + hist * D * 2 * 2 + cfg.context * D * 2 * 2
    step_bytes = per_layer * cfg.layers
    pk, pk_kind = peaks()
    achieved = step_bytes / (ms / 1000.0) / 1e9
    if pg is not None:
        del gather, static, stack
        pg.barrier()
        pg.destroy_process_group()
    if rank != 0:
        return 0
    line = {"metric": "verify_steps_per_s", "value": 1000.0 / ms, "unit": "verify-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8-e4m3 GEMMs, bf16 attention" if args.fp8 else "bf16",
            "data": "synthetic (seeded weights N(0,0.02), random unit-scale KV history)",
            "config": {"workload": "cfg3: 30-layer verify of 4 candidates x 32 action tokens over a "
                                   "read-only 3520-token history, 512 context tokens",
                       "global_batch": B_all, "seq_len": Q, "kv_history": hist, "context": cfg.context,
                       "parallelism": (f"candidates split {B}/GPU, history NCCL-broadcast once, "
                                       "candidate outputs all-gathered each step" if world > 1
                                       else "one GPU"),
                       "history_broadcast": bcast,
                       "l2": "inputs larger than L2 (weights streamed every step)"},
            "roofline": {"kernel": "whole step on one GPU (GEMM weight streaming dominates)", "bound": "hbm",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": None,
                         "peak_source": f"{pk_kind} HBM copy", "algorithmic_bytes_per_step": step_bytes},
            "e2e": {"value": 1000.0 / ms_e2e, "unit": "verify-steps/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": (hx.numel() * 2 + ht.numel() * 4) * world,
                    "d2h_bytes_per_step": hout.numel() * 2 * world,
                    "copies": "each step's inputs copied in from pinned host memory and its output copied out, "
                              "on a copy stream overlapped with the neighbouring steps (PipelinedIO)",
                    "serial_ms_per_step": ms_serial},
            "gpu_launches": NativeStack.launches_per_layer(True, args.fp8) * cfg.layers * args.steps,
            "clocks": clk, "device_error": dev_code}
    print(json.dumps(line), flush=True)
    return 0


def run_action_chunk(args):
    """--workload action_chunk: one FastWAM-style action chunk end to end on
    1 GPU: 10 flow-match updates, each a whole-model forward in action mode
    (action embedding, timestep embedding chain, 30 cfg2 blocks over a
    3520-token read-only KV history with the prepared 512-token text
    context, output norm and projection) and the scheduler step, for 8
    rollouts x 32 action tokens, as one CUDA graph."""
    from wam_ops import _lib, configs
    from wam_ops.model import NativeActionDenoiser, NativeWanModel
    from wam_ops.scheduler import FlowMatchScheduler

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = configs.PRESETS["cfg2"]
    B, steps = 8, 10
    gen = torch.Generator(device=dev).manual_seed(99)
    torch.set_grad_enabled(False)
    model = configs.build_model(cfg, dev, seed=99)
    configs.fill_history(list(model.blocks), cfg, dev, gen, pool_batch=B)
    nm = NativeWanModel(model, fp8=args.fp8)
    text = torch.randn(B, cfg.context, 4096, generator=gen, device=dev).bfloat16()
    nm.prepare_context(text)
    # Cross K/V construction of a new context (text projection + every
    # layer's K/V projection and RMS), timed apart from the chunk: the 8
    # rollouts' own contexts, and the per-chunk rebuild of one context.
    D = cfg.dim

    def time_prepare(t):
        nm.prepare_context(t)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(3):
            nm.prepare_context(t)
        c1.record()
        torch.cuda.synchronize()
        ms_ = c0.elapsed_time(c1) / 3
        rows = t.shape[0] * t.shape[1]
        flops = 2.0 * rows * (4096 * D + D * D) + len(nm.stack.layers) * 2 * 2.0 * rows * D * D
        return {"contexts": t.shape[0], "tokens": t.shape[1], "ms": ms_,
                "tflops": flops / ms_ / 1e9, "gflop": flops / 1e9}
    ctx_one = time_prepare(text[:1].contiguous())
    ctx_all = time_prepare(text)
    ctx_ms = ctx_all["ms"]
    f, h, w = cfg.action
    x = torch.randn(B, 30, f, h, w, generator=gen, device=dev).bfloat16()
    grid = configs.mesh_id(f, h, w, 0, f_shift=cfg.history_chunks, action=True)[None].to(dev)
    sched = FlowMatchScheduler(shift=5.0, sigma_min=0.0, extra_one_step=True)
    sched.set_timesteps(steps)
    den = NativeActionDenoiser(nm, sched)
    den.capture(x, grid)
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)          # the sampler starts; the warm-up then brings the clocks back up
    for _ in range(args.warmup):
        den.run(x)
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError("device error during warm-up")
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        den.run()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    hx = x.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    e0.record(stream)
    for _ in range(args.steps):
        out = den.run(hx.to(dev, non_blocking=True))
        hout.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    line = {"metric": "action_chunks_per_s", "value": B * 1000.0 / ms, "unit": "action-chunks/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 GEMMs, bf16 attention" if args.fp8 else "bf16",
            "data": "synthetic (seeded weights N(0,0.02), random unit-scale KV history and text)",
            "config": {"workload": "action chunk: 10 flow-match updates (shift 5) of the whole model in "
                                   "action mode, 8 rollouts x 32 action tokens, cfg2 blocks (D3072, 30 "
                                   "layers) over a 3520-token KV history, 512 prepared text tokens",
                       "global_batch": B, "seq_len": 32, "kv_history": cfg.history_chunks * cfg.tokens,
                       "denoise_updates_per_chunk": steps, "ms_per_update": ms / steps,
                       "context_prepare_ms": ctx_ms, "context_prepare": [ctx_all, ctx_one]},
            "e2e": {"value": B * 1000.0 / ms_e2e, "unit": "action-chunks/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hout.numel() * 2},
            "gpu_launches": den.launches_per_chunk() * args.steps, "clocks": clk,
            "device_error": _lib.device_status()}
    print(json.dumps(line), flush=True)
    return 0


def _random_draft(dev, channels=7, seed=5):
    """A seeded random-weight FastWAM DirectionPredictor state_dict (the
    reference's names and shapes; no trained checkpoint is available)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    A, E, F = channels, 64, 256
    shapes = {"embed.weight": (E, 2 * A + 3), "embed.bias": (E,), "position": (1, 32, E),
              "block.self_attn.in_proj_weight": (3 * E, E), "block.self_attn.in_proj_bias": (3 * E,),
              "block.self_attn.out_proj.weight": (E, E), "block.self_attn.out_proj.bias": (E,),
              "block.linear1.weight": (F, E), "block.linear1.bias": (F,), "block.linear2.weight": (E, F),
              "block.linear2.bias": (E,), "block.norm1.weight": (E,), "block.norm1.bias": (E,),
              "block.norm2.weight": (E,), "block.norm2.bias": (E,), "head.weight": (2 * A, E),
              "head.bias": (2 * A,)}
    sd = {k: torch.randn(v, generator=g, device=dev) * 0.1 for k, v in shapes.items()}
    for k in ("block.norm1.weight", "block.norm2.weight"):
        sd[k] += 1.0
    n = 2 * 32 * A + 3
    sd.update(feature_mean=torch.zeros(n, device=dev), feature_std=torch.ones(n, device=dev),
              residual_mean=torch.zeros(32 * A, device=dev), residual_std=torch.full((32 * A,), 0.05, device=dev))
    return sd


def run_spec_chunk(args):
    """--workload spec_chunk: one action chunk (10 flow-match updates) of one
    rollout through the speculative K2/B2 loop of the reference
    (fastwam-base/fullcode-v1/real_speculative.py:32-109): the device draft
    predictor proposes a 7-state tree, ONE target forward (the whole model in
    action mode, 30 cfg2 blocks over a 3520-token read-only KV history with
    the prepared 512-token text context, 7 candidate rows) verifies it, the
    device scores and route commit 1-3 updates. Target forwards replay CUDA
    graphs (1 and 7 rows); the draft is random-weight (no trained
    checkpoint), so the line reports the two ends of acceptance: every tree
    accepted at depth 2 (tau above every score; the headline value) and
    every tree rejected (tau 0), beside the plain 10-update chunk."""
    from wam_ops import _lib, configs
    from wam_ops import speculative as sp
    from wam_ops.model import NativeWanModel
    from wam_ops.scheduler import FlowMatchScheduler

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = configs.PRESETS["cfg2"]
    A, steps = 7, 10
    gen = torch.Generator(device=dev).manual_seed(98)
    torch.set_grad_enabled(False)
    model = configs.build_model(cfg, dev, seed=98, action_dim=A)
    configs.fill_history(list(model.blocks), cfg, dev, gen, pool_batch=1)
    nm = NativeWanModel(model)
    nm.prepare_context(torch.randn(1, cfg.context, 4096, generator=gen, device=dev).bfloat16())
    f, h, w = cfg.action
    rope = configs.rope_freqs(configs.mesh_id(f, h, w, 0, f_shift=cfg.history_chunks, action=True)
                              .to(device=dev, dtype=torch.float64))
    target = sp.GraphedTarget(sp.NativeActionTarget(nm, (f, h, w), rope))
    draft = sp.DraftPredictor(_random_draft(dev, A))
    sched = FlowMatchScheduler(shift=5.0, sigma_min=0.0, extra_one_step=True)
    sched.set_timesteps(steps)
    ts = [float(t) for t in sched.timesteps[:steps]]
    ds = [sched.delta(t) for t in sched.timesteps[:steps]]
    state0 = torch.randn(1, 32, A, generator=gen, device=dev).bfloat16()
    times = torch.tensor(ts, dtype=torch.float32, device=dev)
    lib, n = _lib.load(), 32 * A

    def plain():
        x = state0.clone()
        for k in range(steps):
            v = target(x, times[k:k + 1])
            _lib.check(lib.wamb_spec_expand(x.data_ptr(), v.data_ptr(), 0, 1, 1, n, ds[k], x.data_ptr(),
                                            _lib.stream_ptr()))
        return x

    arms = {"accept_all": sp.K2B2Speculative(target, draft, 1e30), "reject_all": sp.K2B2Speculative(target, draft, 0.0)}
    runs = {name: (lambda s=spec: s.loop(state0, ts, ds)) for name, spec in arms.items()}
    runs["plain"] = plain
    for _ in range(args.warmup):
        for r in runs.values():
            r()
    torch.cuda.synchronize()
    if _lib.device_status() != 0:
        raise RuntimeError("device error during warm-up")
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms, clk = {}, None
    for name, r in runs.items():
        clocks = Clocks(0)
        clocks.start()
        time.sleep(0.3)      # the sampler starts; one untimed run brings the clocks back up
        r()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            r()
        e1.record(stream)
        torch.cuda.synchronize()
        c = clocks.stop()
        clk = c if name == "accept_all" else clk
        ms[name] = e0.elapsed_time(e1) / args.steps
    hx = state0.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    e0.record(stream)
    for _ in range(args.steps):
        out = arms["accept_all"].loop(hx.to(dev, non_blocking=True), ts, ds)
        hout.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    calls = {k: len(s.rounds) for k, s in arms.items()}
    per_forward = nm.stack.launches_per_step(with_cache=True) + 12   # blocks + embedders / head
    line = {"metric": "spec_action_chunks_per_s", "value": 1000.0 / ms["accept_all"], "unit": "action-chunks/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms["accept_all"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded model weights N(0,0.02), random unit-scale KV history and text, "
                    "random-weight draft predictor)",
            "config": {"workload": "speculative action chunk (K2/B2): 10 flow-match updates (shift 5) of one "
                                   "rollout, 32 x 7 action tokens, cfg2 blocks (D3072, 30 layers) over a "
                                   "3520-token read-only KV history, 512 prepared text tokens; 7-row tree "
                                   "verification per round",
                       "global_batch": 1, "seq_len": 32, "kv_history": cfg.history_chunks * cfg.tokens,
                       "denoise_updates_per_chunk": steps,
                       "rounds": {k: [r[1] for r in s.rounds] for k, s in arms.items()},
                       "target_forwards_per_chunk": calls,
                       "ms_per_chunk": ms, "plain_chunks_per_s": 1000.0 / ms["plain"],
                       "reject_all_chunks_per_s": 1000.0 / ms["reject_all"],
                       "speedup_accept_all_vs_plain": ms["plain"] / ms["accept_all"]},
            "e2e": {"value": 1000.0 / ms_e2e, "unit": "action-chunks/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hout.numel() * 2},
            # per chunk: target forwards, 7 kernels per tree round (2 draft, 2 expand, scores, route,
            # commit), 1 step per ordinary round
            "gpu_launches": args.steps * sum(per_forward + (7 if r[1] is not None else 1)
                                             for r in arms["accept_all"].rounds),
            "clocks": clk, "device_error": _lib.device_status()}
    print(json.dumps(line), flush=True)
    return 0


def run_kernel_case(args):
    """--workload kernel --case NAME: one kernel (or one block) at a fixed
    shape, 3 warm-up launches then --launches more, for ncu captures (inputs
    larger than L2, a few hundred MB to a few GB on the device). Prints one
    status line; no timing is reported (use the workloads above for that).

    ffn1       FFN1 GEMM + GELU epilogue, M x 14336 x 3072 (--m, cfg2 weights);
               --fp8: E4M3 operands (quantized once before the launches)
    small      small-M GEMM + residual epilogue (the verify batch's O / FFN-out
               projections, --m/--n/--k); 12 weight copies rotate so every
               launch streams its weights from HBM
    res_gate   the O projection (M x 3072 x 3072, gated fp32 residual) beside
               the same GEMM with an ungated residual and bias-only epilogues;
               prints each one's CUDA-event time
    attention  self attention of --batch cfg2 rollouts of --q queries over
               --pool keys (24 heads) with the block's partial scratch: key
               tiles shared over the SMs (stream-K) when whole (query tile
               pair, head, batch row) items would leave SMs idle
    attention_whole  the same call without partial scratch: one item per CTA
               (--kv-splits N > 0 with either: that many key splits on
               attn_tc_kernel instead)
    verify_attention  cfg3 self attention: 4 candidates x 32 queries sharing
               one 3520-slot history row plus their own keys (24 heads)
    quant      row quantization to E4M3 of an --m x --k bf16 matrix
    block      one cfg2-shape block (no cache) of --batch x --q rows: its
               LayerNorm and RMS+RoPE launches are the memory-bound kernels
               to capture (ncu -k regex:ln_kernel / rms_rope_kernel)
    """
    from wam_ops import _lib, configs, ops

    torch.set_grad_enabled(False)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    D, H, F = 3072, 24, 14336
    a = args
    if a.case == "ffn1":
        x = torch.randn(a.m, D, generator=g, device=dev).bfloat16()
        w = (torch.randn(F, D, generator=g, device=dev) * 0.02).bfloat16()
        b = torch.zeros(F, device=dev, dtype=torch.bfloat16)
        out = torch.empty(a.m, F, device=dev, dtype=torch.bfloat16)
        if a.fp8:
            x8, sx = ops.quantize_rows(x)
            w8, sw = ops.quantize_rows(w)
            run = lambda: ops.linear(x8, w8, b, epilogue=_lib.EPI_GELU, out=out,  # noqa: E731
                                     a_scale=sx, w_scales=sw)
        else:
            run = lambda: ops.linear(x, w, b, epilogue=_lib.EPI_GELU, out=out)  # noqa: E731
    elif a.case == "small":
        x = torch.randn(a.m, a.k, generator=g, device=dev).bfloat16()
        ws = [(torch.randn(a.n, a.k, generator=g, device=dev) * 0.02).bfloat16() for _ in range(12)]
        b = torch.zeros(a.n, device=dev, dtype=torch.bfloat16)
        res = torch.randn(a.m, a.n, generator=g, device=dev).bfloat16()
        out = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        it = iter(range(1 << 30))
        run = lambda: ops.linear(x, ws[next(it) % 12], b, epilogue=_lib.EPI_RES, out=out,  # noqa: E731
                                 res=res)
    elif a.case == "res_gate":
        cfg = configs.PRESETS["cfg2"]
        x = torch.randn(a.m, D, generator=g, device=dev).bfloat16()
        w = (torch.randn(D, D, generator=g, device=dev) * 0.02).bfloat16()
        b = torch.zeros(D, device=dev, dtype=torch.bfloat16)
        res = torch.randn(a.m, D, generator=g, device=dev)
        out = torch.empty(a.m, D, device=dev)
        out_bf = torch.empty(a.m, D, device=dev, dtype=torch.bfloat16)
        table = torch.randn(6, D, generator=g, device=dev) / D ** 0.5
        temb = configs.make_temb(cfg, 8, dev, g)
        gate = dict(table=table, temb=temb, rows_per_batch=a.m // 8, gate_index=2)
        run = lambda: ops.linear(x, w, b, epilogue=_lib.EPI_RES_GATE, out=out, res=res, **gate)  # noqa: E731
        variants = (("res_gate", run),
                    ("res_f32", lambda: ops.linear(x, w, b, epilogue=_lib.EPI_RES, out=out, res=res)),
                    ("bias_f32", lambda: ops.linear(x, w, b, out=out)),
                    ("bias_bf16", lambda: ops.linear(x, w, b, out=out_bf)))
        for name, f in variants:
            for _ in range(3):
                f()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                f()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 20 * 1e3
            print(f"{name}: {us:.1f} us, {2.0 * a.m * D * D / us / 1e6:.1f} TFLOP/s")
    elif a.case == "verify_attention":
        B, Q, pool, hist = 4, 32, 4400, 3520
        kp = torch.randn(2 * pool, D, generator=g, device=dev).bfloat16()
        vp = torch.randn(2 * pool, D, generator=g, device=dev).bfloat16()
        qkv = torch.randn(B * Q, 3 * D, generator=g, device=dev).bfloat16()
        tl = [(s0, min(128, hist - s0)) for s0 in range(0, hist, 128)]
        tiles = torch.tensor(tl, dtype=torch.int32, device=dev).view(-1, 2)
        n = torch.tensor([len(tl)], dtype=torch.int32, device=dev)
        rows = torch.zeros(B, dtype=torch.int64, device=dev)
        out = torch.empty(B * Q, D, device=dev, dtype=torch.bfloat16)
        run = lambda: ops.attention(qkv, kp, vp, heads=H, q_rows=Q, src0_batch_stride=pool,  # noqa: E731
                                    tiles=tiles, n_tiles=n, src0_map=rows, k1=qkv, v1=qkv, k1_col=D,
                                    v1_col=2 * D, out=out)
    elif a.case in ("attention", "attention_whole"):
        q = torch.randn(a.batch * a.q, D, generator=g, device=dev).bfloat16()
        kp = torch.randn(a.batch * a.pool, D, generator=g, device=dev).bfloat16()
        vp = torch.randn(a.batch * a.pool, D, generator=g, device=dev).bfloat16()
        out = torch.empty(a.batch * a.q, D, device=dev, dtype=torch.bfloat16)
        ks = a.kv_splits if a.kv_splits > 0 else (0 if a.case == "attention" else None)
        run = lambda: ops.attention(q, kp, vp, heads=H, q_rows=a.q, src0_batch_stride=a.pool,  # noqa: E731
                                    src0_len=a.pool, out=out, kv_splits=ks)
    elif a.case == "quant":
        x = torch.randn(a.m, a.k, generator=g, device=dev).bfloat16()
        run = lambda: ops.quantize_rows(x)  # noqa: E731
    else:
        cfg = configs.PRESETS["cfg2"]
        blk = configs.build_blocks(configs.Config("p", D, H, F, 1, 1, (1, 16, 53), (8, 4, 1), 8), dev)[0]
        from wam_ops.native import NativeBlock
        nb = NativeBlock(blk, fp8=a.fp8)
        x = torch.randn(a.batch, a.q, D, generator=g, device=dev).bfloat16()
        ctx = torch.randn(1, 8, D, generator=g, device=dev).bfloat16()
        temb = configs.make_temb(cfg, a.batch, dev, g)
        rope = configs.rope_freqs(torch.zeros(3, a.q)).to(dev)
        run = lambda: nb(x, ctx, temb, rope)  # noqa: E731
    for _ in range(3 + a.launches):
        run()
    torch.cuda.synchronize()
    code = _lib.device_status()
    print(f"{a.case}: ok, device status {code}")
    return 0 if code == 0 else 1


def stack_flops(cfg, split=False):
    """Algorithmic FLOPs of one 30-layer step for ONE rollout: the six
    projections, the two FFN GEMMs and the QK^T / PV products of both
    attentions (cross K/V prepared, not counted). split=True returns
    (GEMM FLOPs, attention FLOPs)."""
    D, F, Q, C = cfg.dim, cfg.ffn, cfg.tokens, cfg.context
    keys = cfg.history_chunks * Q + Q
    proj = 2 * Q * D * (3 * D) + 2 * Q * D * D + 2 * Q * D * D + 2 * Q * D * D
    ffn = 2 * 2 * Q * D * F
    attn = 2 * 2 * Q * keys * D + 2 * 2 * Q * C * D
    if split:
        return cfg.layers * (proj + ffn), cfg.layers * attn
    return cfg.layers * (proj + ffn + attn)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--step-only", action="store_true",
                    help="default workload: time the bf16 step only (for ncu launch lists)")
    ap.add_argument("--fp8", action="store_true",
                    help="E4M3 GEMMs (the FP8 weight path); default is the bf16 drop-in")
    ap.add_argument("--case", default="ffn1",
                    choices=["ffn1", "small", "res_gate", "attention", "attention_whole", "verify_attention", "quant",
                             "block"],
                    help="--workload kernel: which single-kernel case to launch (for ncu captures)")
    ap.add_argument("--m", type=int, default=2048)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=14336)
    ap.add_argument("--q", type=int, default=880)
    ap.add_argument("--pool", type=int, default=4400)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--launches", type=int, default=1)
    ap.add_argument("--kv-splits", type=int, default=0,
                    help="--case attention: a forced key-split factor for attn_tc_kernel (0: the library's choice)")
    ap.add_argument("--workload", default="cfg4",
                    choices=["cfg4", "cfg3", "cfg2", "cfg1", "action_chunk", "spec_chunk", "kernel"],
                    help="cfg4 (default, the headline): 8 cfg2 rollouts per GPU; cfg3: the "
                         "4 x 32-token candidate verify step on one GPU; action_chunk: 10 whole-model "
                         "denoise updates of an action chunk; spec_chunk: the same chunk for one rollout "
                         "through the speculative K2/B2 loop")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "cfg3":
        return run_verify(args)
    if args.workload == "action_chunk":
        return run_action_chunk(args)
    if args.workload == "spec_chunk":
        return run_spec_chunk(args)
    if args.workload == "kernel":
        return run_kernel_case(args)
    if args.workload in ("cfg2", "cfg1"):
        return run_config(args)
    return run_native(args)


if __name__ == "__main__":
    sys.exit(main())
