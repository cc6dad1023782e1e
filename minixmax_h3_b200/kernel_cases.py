"""Single-kernel cases for profiling and timing sweeps.

    python -m minixmax_h3_b200.kernel_cases attention --seq 131072 --heads 3 [--layout packed]
    python -m minixmax_h3_b200.kernel_cases gemm_nvfp4 --m 8192 --n 9216 --k 3072 [--epi gelu]
    python -m minixmax_h3_b200.kernel_cases gemm_i8 --m 8192 --n 9216 --k 3072
    python -m minixmax_h3_b200.kernel_cases gemm_sweep --warmup 3 --iters 20   # cfg 2 + cfg 3 shapes, M 32768
    python -m minixmax_h3_b200.kernel_cases quant_nvfp4 --m 32768 --k 3072
    python -m minixmax_h3_b200.kernel_cases quant_nvfp4 --m 32768 --k 12288 --epi gelu   # GELU on load
    python -m minixmax_h3_b200.kernel_cases quant_i8 --m 32768 --k 3072
    python -m minixmax_h3_b200.kernel_cases quant_i8_convrot --m 32768 --k 3072
    python -m minixmax_h3_b200.kernel_cases qk_rope --seq 131072 --heads 24
    python -m minixmax_h3_b200.kernel_cases rmsnorm_modulate --m 131072 --k 3072
    python -m minixmax_h3_b200.kernel_cases rmsnorm_modulate_quant_i8 --m 32768 --k 3072
    python -m minixmax_h3_b200.kernel_cases rmsnorm_modulate_quant_i8_convrot --m 32768 --k 3072
    python -m minixmax_h3_b200.kernel_cases exchange_2gpu --m 8192 --heads 24 --k 3072   # needs 2 GPUs

Each case allocates its inputs once, launches the kernel `--warmup` times,
then `--iters` times between CUDA events on the launching stream, and prints
one JSON line (ms per launch and the algorithmic throughput).  Inputs are
synthetic N(0,1) (weights N(0,0.02)).  Sizes are chosen by the caller so a
profiler capture stays small.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / max(iters, 1)


SWEEP_KN = ((3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072))


EPILOGUES = {"store": ops.EPI_STORE, "gelu": ops.EPI_GELU, "gate_res": ops.EPI_GATE_RES}


def _gemm(case: str, m: int, n: int, k: int, warmup: int, iters: int, g, dev, epi: str = "store") -> dict:
    x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    kw: dict = {"epilogue": EPILOGUES[epi], "out": out}
    if epi == "gate_res":  # out += gate[row_sel] * y, adaLN rows 0/1 as in the block
        kw.update(resid=out, gate=(0.1 * torch.randn(2, n, generator=g, device=dev)).to(torch.bfloat16),
                  row_sel=(torch.arange(m, device=dev) < 512).to(torch.int32))
    if case == "gemm_nvfp4":
        xa, wq = ops.quant_nvfp4(x), ops.quant_nvfp4(w)
        ms = _time(lambda: ops.gemm_nvfp4(xa, wq, **kw), warmup, iters)
    else:
        q, xs = ops.quant_i8_rows(x)
        wq = torch.randint(-128, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
        ws = torch.rand(n, device=dev, generator=g) * 1e-3
        ms = _time(lambda: ops.gemm_i8(q, xs, wq, ws, **kw), warmup, iters)
    flops = 2.0 * m * n * k
    return {"m": m, "n": n, "k": k, "epilogue": epi, "ms": ms, "tflops": flops / ms / 1e9, "flops": flops}


def _exchange_2gpu(s_local: int, heads: int, hidden: int, warmup: int, iters: int, g, dev) -> None:
    """Rank 0 of a 2-rank Ulysses group, both GPUs driven by this one process:
    the QKV GEMM with the seq->head scatter fused into its epilogue and the
    attention with the head->seq scatter, each against the same kernel
    writing locally.  Half of each fused output crosses NVLink (peer access
    enabled between the two devices; no kernel waits on the other GPU)."""
    from cuda.bindings import runtime as rt

    if torch.cuda.device_count() < 2:
        raise SystemExit("exchange_2gpu needs 2 GPUs")
    peer = torch.device("cuda", 1)
    torch.cuda.set_device(dev)
    (err,) = rt.cudaDeviceEnablePeerAccess(1, 0)
    if err not in (rt.cudaError_t.cudaSuccess, rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
        raise SystemExit(f"cudaDeviceEnablePeerAccess: {err}")
    hl, s = heads // 2, 2 * s_local
    # QKV projection of this rank's s_local tokens
    x = torch.randn(s_local, hidden, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(3 * heads * 128, hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    xa, wq = ops.quant_nvfp4(x), ops.quant_nvfp4(w)
    recv = [torch.zeros(s, 3, hl, 128, dtype=torch.bfloat16, device=d) for d in (dev, peer)]
    y = torch.empty(s_local, 3 * heads * 128, dtype=torch.bfloat16, device=dev)
    flops = 2.0 * s_local * w.shape[0] * hidden
    ms_plain = _time(lambda: ops.gemm_nvfp4(xa, wq, out=y), warmup, iters)
    ms_fused = _time(lambda: ops.gemm_nvfp4_seq2head(xa, wq, None, [r.data_ptr() for r in recv], 0, heads),
                     warmup, iters)
    peer_bytes = s_local * 3 * hl * 128 * 2
    print(json.dumps({"case": "gemm_nvfp4_seq2head", "m": s_local, "n": w.shape[0], "k": hidden,
                      "ms_plain": ms_plain, "ms_fused": ms_fused, "tflops_fused": flops / ms_fused / 1e9,
                      "peer_bytes": peer_bytes, "peer_gbs": peer_bytes / ms_fused / 1e6}), flush=True)
    # attention over this rank's heads of all s tokens, rows scattered to the token owners
    q, k, v = (torch.randn(s, hl, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    o_plain = torch.empty(s, hl, 128, dtype=torch.bfloat16, device=dev)
    outs = [torch.zeros(s_local, heads, 128, dtype=torch.bfloat16, device=d) for d in (dev, peer)]
    aflops = 4.0 * s * s * 128 * hl
    ms_plain = _time(lambda: ops.attention(q, k, v, out=o_plain), warmup, iters)
    ms_fused = _time(lambda: ops.attention_head2seq(q, k, v, [o.data_ptr() for o in outs], s_local=s_local, head0=0,
                                                    total_heads=heads), warmup, iters)
    peer_bytes = s_local * hl * 128 * 2
    print(json.dumps({"case": "attention_head2seq", "seq": s, "heads": hl, "ms_plain": ms_plain,
                      "ms_fused": ms_fused, "tflops_fused": aflops / ms_fused / 1e9, "peer_bytes": peer_bytes,
                      "peer_gbs": peer_bytes / ms_fused / 1e6}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=["attention", "gemm_nvfp4", "gemm_i8", "quant_nvfp4", "quant_i8",
                                       "quant_i8_convrot", "qk_rope", "rmsnorm_modulate", "rmsnorm_modulate_quant_i8",
                                       "rmsnorm_modulate_quant_i8_convrot", "gemm_sweep", "exchange_2gpu"])
    ap.add_argument("--seq", type=int, default=16384)
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=9216)
    ap.add_argument("--k", type=int, default=3072)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--epi", choices=sorted(EPILOGUES), default="store",
                    help="GEMM epilogue; with quant_nvfp4, gelu quantises gelu(x) (the MLP fc2 input)")
    ap.add_argument("--layout", choices=["separate", "packed"], default="separate",
                    help="attention: separate [S, H, 128] tensors or views of a packed [S, 3, H, 128] QKV")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    rec: dict = {"case": a.case}
    if a.case == "attention":
        if a.layout == "packed":  # q/k/v as views of one [S, 3, H, 128] projection output, as in a block
            qkv = torch.randn(a.seq, 3, a.heads, 128, generator=g, device=dev).to(torch.bfloat16)
            q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        else:
            q, k, v = (torch.randn(a.seq, a.heads, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        o = torch.empty(a.seq, a.heads, 128, dtype=torch.bfloat16, device=dev)
        ms = _time(lambda: ops.attention(q, k, v, out=o), a.warmup, a.iters)
        flops = 4.0 * a.seq * a.seq * 128 * a.heads
        rec.update(seq=a.seq, heads=a.heads, ms=ms, tflops=flops / ms / 1e9, flops=flops)
    elif a.case in ("gemm_nvfp4", "gemm_i8"):
        rec.update(_gemm(a.case, a.m, a.n, a.k, a.warmup, a.iters, g, dev, a.epi))
    elif a.case == "gemm_sweep":
        # BASELINE cfg 2 / cfg 3: M = 32768 tokens, (K, N) of the four projections
        m = a.m if a.m != ap.get_default("m") else 32768
        for case in ("gemm_i8", "gemm_nvfp4"):
            for k, n in SWEEP_KN:
                print(json.dumps({"case": case, **_gemm(case, m, n, k, a.warmup, a.iters, g, dev, a.epi)}), flush=True)
        return
    elif a.case == "exchange_2gpu":
        _exchange_2gpu(a.m, a.heads, a.k, a.warmup, a.iters, g, dev)
        return
    elif a.case == "qk_rope":
        # q and k views of a packed [S, 3, H, 128] QKV buffer, in place
        from .block import RopeSpec
        qkv = torch.randn(a.seq, 3, a.heads, 128, generator=g, device=dev).to(torch.bfloat16)
        w = torch.ones(128, dtype=torch.bfloat16, device=dev)
        side = int(round((a.seq / 4) ** 0.5))
        t_len = (a.seq + side * side - 1) // (side * side)
        pos = RopeSpec.grid_positions(t_len, side, side)[: a.seq]
        rope = RopeSpec.build(pos, device=dev)
        ms = _time(lambda: ops.qk_rmsnorm_rope(qkv[:, 0], qkv[:, 1], w, w, 1e-6, rope.pos, 0, rope.inv_freq,
                                               rope.n_t, rope.n_h), a.warmup, a.iters)
        nbytes = 2 * 2 * a.seq * a.heads * 128 * 2 + a.seq * 3 * 4  # q, k read + written; positions
        rec.update(seq=a.seq, heads=a.heads, ms=ms, gbs=nbytes / ms / 1e6, bytes=nbytes)
    elif a.case.startswith("rmsnorm_modulate_quant_i8"):
        x = torch.randn(a.m, a.k, generator=g, device=dev).to(torch.bfloat16)
        w = torch.ones(a.k, dtype=torch.bfloat16, device=dev)
        tab = (torch.randn(2, 2 * a.k, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        row_sel = torch.zeros(a.m, dtype=torch.int32, device=dev)
        q = torch.empty(a.m, a.k, dtype=torch.int8, device=dev)
        xs = torch.empty(a.m, dtype=torch.float32, device=dev)
        group = 256 if a.case.endswith("convrot") else 0
        ms = _time(lambda: ops.rmsnorm_modulate_quant_i8(x, w, tab[:, : a.k], tab[:, a.k:], 1e-6, row_sel=row_sel,
                                                         convrot_group=group, q_out=q, scale_out=xs),
                   a.warmup, a.iters)
        nbytes = 2 * a.m * a.k + a.m * a.k + 4 * a.m + 4 * a.m  # x read, codes, row scales, row indices
        rec.update(m=a.m, k=a.k, ms=ms, gbs=nbytes / ms / 1e6, bytes=nbytes)
    elif a.case == "rmsnorm_modulate":
        x = torch.randn(a.m, a.k, generator=g, device=dev).to(torch.bfloat16)
        w = torch.ones(a.k, dtype=torch.bfloat16, device=dev)
        tab = (torch.randn(2, 2 * a.k, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        row_sel = torch.zeros(a.m, dtype=torch.int32, device=dev)
        out = torch.empty_like(x)
        amax = torch.zeros(1, dtype=torch.float32, device=dev)
        ms = _time(lambda: ops.rmsnorm_modulate(x, w, tab[:, : a.k], tab[:, a.k:], 1e-6, row_sel=row_sel, out=out,
                                                amax_out=amax), a.warmup, a.iters)
        nbytes = 2 * a.m * a.k * 2 + 4 * a.m  # x read, h written, row indices
        rec.update(m=a.m, k=a.k, ms=ms, gbs=nbytes / ms / 1e6, bytes=nbytes)
    else:
        x = torch.randn(a.m, a.k, generator=g, device=dev).to(torch.bfloat16)
        if a.case == "quant_nvfp4" and a.epi == "gelu":
            # fc2's input quantiser with the MLP's GELU applied on load (x plays fc1's output y)
            ymax2 = torch.zeros(2, dtype=torch.float32, device=dev)
            ymax2[0] = x.float().max().clamp(min=0.0)
            ops.gelu_amax_scan(x, ymax2)
            ms = _time(lambda: ops.quant_nvfp4_gelu(x, ymax2), a.warmup, a.iters)
            nbytes = 2 * a.m * a.k + a.m * a.k // 2 + a.m * a.k // 16
        elif a.case == "quant_nvfp4":
            amax = ops.amax(x)
            ms = _time(lambda: ops.quant_nvfp4(x, amax_t=amax), a.warmup, a.iters)
            nbytes = 2 * a.m * a.k + a.m * a.k // 2 + a.m * a.k // 16
        else:
            group = 256 if a.case == "quant_i8_convrot" else 0
            ms = _time(lambda: ops.quant_i8_rows(x, convrot_group=group), a.warmup, a.iters)
            nbytes = 3 * a.m * a.k + 4 * a.m
        rec.update(m=a.m, k=a.k, ms=ms, gbs=nbytes / ms / 1e6, bytes=nbytes)
    print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
