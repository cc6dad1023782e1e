"""Benchmark: one denoising step of four MiniMax-H3 DiT blocks (BASELINE cfg 5).

Workload (the same total sequence at every N — strong scaling):
  hidden 3072, 24 heads x 128, GELU MLP 12288, NVFP4 W4A4 for every linear,
  512 text tokens (dim 4096, through condition_proj) + 497,760 video tokens
  (grid t61 x h68 x w120) = 498,272 tokens of joint attention, 3D RoPE
  44/42/42, adaLN from a 256-d sinusoidal timestep embedding.  Random-init
  weights (no checkpoints offline), synthetic bf16 N(0,1) inputs; every
  activation tensor (3 GB and up) is far larger than the 126 MB L2.
  N > 1: Ulysses sequence parallelism over NCCL, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    (N > 1: torchrun --nproc-per-node N bench.py --gpus N ...)

One JSON line on rank 0.  `value` = block-tokens/s (S x blocks / step time)
with inputs resident in HBM; `e2e` = the same through the public API with the
step's inputs copied from pinned host memory and its output read back inside
the timed region.  `roofline` covers the dominant kernel (flash attention),
timed live with CUDA events around its launches during the timed steps.
`--impl reference` times the reference's CPU torch path (restated by the
oracle, since the reference tree does not travel) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, HEADS, FFN, DEPTH, TEXT_DIM, N_TEXT = 3072, 24, 12288, 4, 4096, 512
GRID = (61, 68, 120)
S_VIDEO = GRID[0] * GRID[1] * GRID[2]
S_TOTAL = N_TEXT + S_VIDEO  # 498,272
METRIC = "DiT-block tokens/s"
REF_TOKENS, REF_Q_ROWS = 1024, 128  # CPU sample per reference step (~1 s of CPU work)
ATTN_DRAM_BYTES_24_HEADS = 1.57e12 + 3.31e9  # ncu dram__bytes_read.sum + write.sum, one launch
UNIT = "block-tokens/s"
WORKLOAD = ("cfg5: one denoising step of 4 DiT blocks, hidden 3072, 24x128 heads, GELU MLP 12288, NVFP4 W4A4 "
            "linears, 512 text (dim 4096) + 497760 video tokens (t61 x h68 x w120) = 498272-token joint attention, "
            "RoPE 44/42/42, Ulysses over N GPUs")


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": d.get("bf16_tflops_sustained", 1385.2), "bf16_burst": d.get("bf16_tflops", 1645.3),
                "hbm": d.get("hbm_gbs", 6535.4), "source": "measured"}
    return {"bf16": 1400.0, "bf16_burst": 1590.0, "hbm": 6650.0, "source": "fallback"}


def positions() -> torch.Tensor:
    """[S_TOTAL, 3] (t, h, w): text token i at (i, 0, 0), then the video grid."""
    from minixmax_h3_b200.block import RopeSpec

    text = torch.stack([torch.arange(N_TEXT, dtype=torch.float32), torch.zeros(N_TEXT), torch.zeros(N_TEXT)], -1)
    return torch.cat([text, RopeSpec.grid_positions(*GRID)])


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU (reference) leg


_CPU_WEIGHTS: dict = {}


def cpu_reference_sample(q_rows: int, lin_tokens: int, seed: int = 0) -> dict:
    """Times the reference's CPU torch path for one block on a bounded sample
    and extrapolates to block-tokens/s at S = 498,272.

    The path is the reference's host code as restated by the oracle: bf16
    RMSNorm/modulate, W4A16 projections (NVFP4 weights decoded to bf16, then
    F.linear — ops/nvfp4.py:154-173), q/k RMSNorm+RoPE (ops/rope.py), SDPA
    attention in bf16 (ops/attention.py:115-117), GELU MLP, gate residuals.
    Sample: `lin_tokens` tokens through everything but attention, plus
    `q_rows` query rows of one head against the full 498,272-token K/V.
    """
    from oracle import h3_oracle as O
    import torch.nn.functional as F

    deq = _CPU_WEIGHTS.get(seed)
    if deq is None:
        g = torch.Generator().manual_seed(seed)
        deq = {}
        for n, (o, i) in {"qkv": (3 * HIDDEN, HIDDEN), "out": (HIDDEN, HIDDEN), "fc1": (FFN, HIDDEN),
                          "fc2": (HIDDEN, FFN)}.items():
            # one-time weight decode, cached like the reference does (modules/linear.py:103)
            w = (torch.randn(o, i, generator=g) * 0.02).to(torch.bfloat16)
            qz = O.nvfp4_quantize(w, hi_first=True)
            deq[n] = O.nvfp4_dequantize(qz["codes"], qz["gs"], qz["sf"], i).to(torch.bfloat16)
        _CPU_WEIGHTS[seed] = deq
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(lin_tokens, HIDDEN, generator=g).to(torch.bfloat16)
    nw = torch.ones(HIDDEN, dtype=torch.bfloat16)
    shift = (0.02 * torch.randn(1, HIDDEN, generator=g)).to(torch.bfloat16)
    scale = (0.02 * torch.randn(1, HIDDEN, generator=g)).to(torch.bfloat16)
    pos = positions()[:lin_tokens]
    table = O.rope_rotation_table(O.rope_angles(pos, O.rope_inv_freq(), 22, 21), torch.bfloat16)
    qw = torch.ones(128, dtype=torch.bfloat16)

    t0 = time.perf_counter()
    h = O.mod_scale_shift(O.rms_norm(x, nw, 1e-6), shift, scale, [(0, lin_tokens, 0)])
    qkv = F.linear(h, deq["qkv"])
    q, k, _v = qkv.view(lin_tokens, 3, HEADS, 128).unbind(1)
    O.rms_rope_apply(q[None], table, qw, 1e-6, 128)
    O.rms_rope_apply(k[None], table, qw, 1e-6, 128)
    o = F.linear(h, deq["out"])
    x = O.mod_gate(x, shift, o, [(0, lin_tokens, 0)])
    h = O.mod_scale_shift(O.rms_norm(x, nw, 1e-6), shift, scale, [(0, lin_tokens, 0)])
    u = F.gelu(F.linear(h, deq["fc1"]))
    x = O.mod_gate(x, shift, F.linear(u, deq["fc2"]), [(0, lin_tokens, 0)])
    t_lin = time.perf_counter() - t0

    qa = torch.randn(1, 1, q_rows, 128, generator=g).to(torch.bfloat16)
    kv = torch.randn(1, 1, S_TOTAL, 128, generator=g).to(torch.bfloat16)
    t0 = time.perf_counter()
    F.scaled_dot_product_attention(qa, kv, kv, scale=128 ** -0.5)
    t_attn = time.perf_counter() - t0

    t_block = t_lin / lin_tokens * S_TOTAL + t_attn / q_rows * S_TOTAL * HEADS
    return {"value": S_TOTAL / t_block, "seconds": t_lin + t_attn,
            "sample": (f"{lin_tokens} tokens through norms/modulation/RoPE/W4A16 projections/GELU MLP + {q_rows} "
                       f"query rows x 1 head of bf16 SDPA against all {S_TOTAL} keys, extrapolated linearly to "
                       f"one block over S={S_TOTAL} ({HEADS} heads)")}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 alone times the CPU path; other ranks exit without work
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    cores = torch.get_num_threads()
    for _ in range(args.warmup):
        cpu_reference_sample(REF_Q_ROWS, REF_TOKENS)
    vals, secs, sample = [], 0.0, ""
    for _ in range(args.steps):
        r = cpu_reference_sample(REF_Q_ROWS, REF_TOKENS)
        vals.append(r["value"])
        secs += r["seconds"]
        sample = r["sample"]
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * S_TOTAL * DEPTH / value,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (W4A16 host path)",
            "data": "synthetic", "config": {"workload": WORKLOAD, "seq_len": S_TOTAL, "blocks": DEPTH},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU leg


def run_gpu(args) -> None:
    import torch.distributed as tdist

    from minixmax_h3_b200 import _lib
    from minixmax_h3_b200 import dist as hdist
    from minixmax_h3_b200.block import ATTN_TIMER, DiTStep, RopeSpec

    st = hdist.init(timeout_s=600.0)
    ws, rank = st.world_size, st.rank
    if ws != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    dev = torch.device("cuda", st.local_rank)
    torch.cuda.set_device(dev)
    _lib.lib()

    step = DiTStep(hidden=HIDDEN, heads=HEADS, ffn=FFN, depth=DEPTH, text_dim=TEXT_DIM, fmt="nvfp4",
                   mlp_act="gelu", device=dev)
    step.init_random(seed=0)  # identical weights on every rank
    rope = RopeSpec.build(positions(), device=dev)
    s_local = S_TOTAL // ws
    s0 = rank * s_local
    n_text_here = max(0, min(N_TEXT, s0 + s_local) - s0)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    video = torch.randn(s_local - n_text_here, HIDDEN, generator=gen, device=dev).to(torch.bfloat16)
    text = torch.randn(N_TEXT, TEXT_DIM, generator=torch.Generator(device=dev).manual_seed(7), device=dev
                       ).to(torch.bfloat16)
    timestep = torch.tensor([500.0], device=dev)
    # host copies for the end-to-end leg (pinned)
    video_h = video.cpu().pin_memory()
    text_h = text.cpu().pin_memory()
    ts_h = timestep.cpu().pin_memory()
    out_h = torch.empty((s_local, HIDDEN), dtype=torch.bfloat16).pin_memory()
    h2d = video_h.numel() * 2 + text_h.numel() * 2 + ts_h.numel() * 4
    d2h = out_h.numel() * 2

    def barrier():
        if ws > 1:
            tdist.barrier(device_ids=[dev.index])

    with torch.no_grad():
        for _ in range(args.warmup):
            step(video, text, timestep, rope)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        launches0 = _lib.LAUNCHES[0]
        ATTN_TIMER.enabled = True
        with ClockSampler(dev.index) as clocks:
            for i in range(args.steps):
                e = ev[i]
                e[0].record()
                video.copy_(video_h, non_blocking=True)  # end-to-end: inputs from pinned host memory
                text.copy_(text_h, non_blocking=True)
                timestep.copy_(ts_h, non_blocking=True)
                e[1].record()
                out = step(video, text, timestep, rope)  # compute on HBM-resident inputs
                e[2].record()
                out_h.copy_(out, non_blocking=True)  # end-to-end: result read back
                e[3].record()
            torch.cuda.synchronize()
            barrier()
            torch.cuda.synchronize()
        ATTN_TIMER.enabled = False
        attn = ATTN_TIMER.drain()
        launches = _lib.LAUNCHES[0] - launches0
    step_ms = [e[1].elapsed_time(e[2]) for e in ev]
    compute_ms = sum(step_ms) / args.steps
    e2e_ms = sum(e[0].elapsed_time(e[3]) for e in ev) / args.steps
    t = torch.tensor([compute_ms, e2e_ms], device=dev)
    if ws > 1:
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    compute_ms, e2e_ms = t.tolist()
    attn_ms = statistics.mean(a for a, _ in attn)
    attn_flops = attn[0][1]
    pk = peaks()
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12
    clock = clocks.summary()
    if rank == 0:
        # DRAM bytes of one full-size attention launch (S = 498,272, 24 heads),
        # from the 1-pass ncu capture in profiles/attention_kernel_S131072_H3.md;
        # a rank's launch covers HEADS/ws heads of the same sequence.
        traffic = ATTN_DRAM_BYTES_24_HEADS * (HEADS // ws) / HEADS
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
            cpu_reference_sample(REF_Q_ROWS, REF_TOKENS)  # warm (weight decode, allocator)
            rs = [cpu_reference_sample(4 * REF_Q_ROWS, 4 * REF_TOKENS) for _ in range(3)]
            cpu = {"value": statistics.mean(r["value"] for r in rs), "unit": UNIT, "cores": torch.get_num_threads(),
                   "kind": "port", "sample": "mean of 3 x " + rs[0]["sample"]}
        line = {
            "metric": METRIC, "value": S_TOTAL * DEPTH / (compute_ms * 1e-3), "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": compute_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4 (e2m1/e4m3) GEMMs + bf16 attention",
            "data": "synthetic (random-init weights, N(0,1) bf16 inputs)",
            "config": {"workload": WORKLOAD, "seq_len": S_TOTAL, "blocks": DEPTH, "hidden": HIDDEN, "heads": HEADS,
                       "mlp": FFN, "parallelism": f"ulysses{ws}", "l2": "inputs larger than L2 (>= 3 GB tensors)"},
            "e2e": {"value": S_TOTAL * DEPTH / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"kernel": "attention_kernel (tcgen05 flash attention)", "bound": "tensor",
                         "achieved": achieved, "peak": pk["bf16"], "unit": "TFLOP/s", "frac": achieved / pk["bf16"],
                         "peak_kind": f"bf16 sustained ({pk['source']})", "traffic": traffic,
                         "launch_ms": attn_ms, "flops_per_launch": attn_flops},
            "cpu_baseline": cpu,
            "clocks": clock,
            "gpu_launches": launches,
            "step_ms": [round(v, 1) for v in step_ms],
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        barrier()
    hdist.destroy()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU leg (quick runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
