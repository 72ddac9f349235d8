"""Benchmark: 14B causal-fast DiT chunk-forward (one denoising step through all blocks) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4] [--impl lbw|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N   (sequence parallel)

Workload (benchmark configuration c4, the headline): 40 blocks of the 14B geometry (dim 5120, 40 heads,
FFN 13824), one 720p chunk of 3 latent frames (45 x 80 tokens per frame, 10,800 query tokens) against a
21-frame KV window (6 cached chunks + the destination chunk = 75,600 keys), 512 text tokens, hoisted
camera FiLM, MXFP8 FFN. Synthetic seeded data with the benchmark distributions (no checkpoints here).
A step = one forward of the whole block stack over the chunk; N ranks shard the query tokens (strong
scaling) and all-gather each block's new K/V over NVLink (copy engines, CUDA IPC buffers).

Printed JSON (rank 0): value = query tokens / step time (max over ranks), e2e = the same through host
buffers (pinned H2D of x, D2H of the result), roofline of the dominant kernel (self-attention), the CPU
baseline (the oracle port timed on a bounded sample on the host cores), clocks sampled during the
timed region, and (after the timed region) the parity of the stack's first block against the CPU oracle on a
sample of query rows.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ATTN_TRAFFIC_C4_BYTES = 2101.592576e6 + 137.902848e6  # ncu dram bytes, one chunk_attn_kernel launch at c4 (tail schedule)
ATTN_KV_BYTES_C4 = 4.0 * 75600 * 5120

CONFIGS = {
    # name: (model, frames, grid_h, grid_w, lead chunks, start_frame, layers override)
    "c1": dict(model="1.3B", grid=(3, 30, 52), n_lead=2, start_frame=6, layers=1),
    "c2": dict(model="14B", grid=(3, 30, 52), n_lead=6, start_frame=18, layers=1),
    "c3": dict(model="1.3B", grid=(3, 30, 52), n_lead=6, start_frame=18, layers=30),
    "c4": dict(model="14B", grid=(3, 45, 80), n_lead=6, start_frame=18, layers=40),
}
TEXT_LEN = 512


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def flops_per_block(lq, lkv, dim, ffn, text=TEXT_LEN):
    bf16 = 8 * lq * dim * dim + 4 * lq * lkv * dim + 4 * lq * dim * dim + 4 * lq * text * dim
    mx = 4 * lq * dim * ffn
    return bf16, mx


class Clocks:
    """nvidia-smi sampler for the timed region (clocks, power, throttle reasons)."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        load = [r[0] for r in rows if r[0] > 0.5 * r[1]] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def config_of(args, world):
    """The `config` object both arms print (the same dict, so the two lines name the same workload)."""
    c = CONFIGS[args.config]
    m = MODELS[c["model"]]
    f, gh, gw = c["grid"]
    chunk = f * gh * gw
    return {"workload": args.config, "model": c["model"], "blocks": c["layers"], "dim": m["dim"],
            "heads": m["num_heads"], "ffn_dim": m["ffn_dim"], "query_tokens": chunk,
            "kv_tokens": (c["n_lead"] + 1) * chunk, "text_tokens": TEXT_LEN, "parallelism": f"sp{world}",
            "lin_mx": bool(getattr(args, "lin_mx", False)),
            "l2": "inputs larger than L2 (KV cache and weights >> 126 MB)"}


# wan/configs/wan_i2v_1_3B.py:21-33 and wan_i2v_A14B.py:16-33 (the same table as lbw_b200.model.CONFIGS; kept here
# so that the CPU reference arm does not load the CUDA package)
MODELS = {"1.3B": dict(dim=1536, ffn_dim=8960, num_heads=12), "14B": dict(dim=5120, ffn_dim=13824, num_heads=40)}


def cpu_oracle_step(cfg_name, rows_sample, threads, blocks=1, mx=False):
    """One block of the oracle (CPU restatement of the reference block) at the workload's geometry on a
    sample of the query rows; returns seconds. mx=False times the bf16 FFN: the reference has no CPU MX path,
    so its CPU block runs the FFN in bf16 (the MX emulation is a parity checker, not a timed baseline)."""
    from oracle import block as ob
    torch.set_num_threads(threads)
    c = CONFIGS[cfg_name]
    m = MODELS[c["model"]]
    C, H, F = m["dim"], m["num_heads"], m["ffn_dim"]
    f, gh, gw = c["grid"]
    chunk = f * gh * gw
    g = torch.Generator().manual_seed(0)
    bf = torch.bfloat16
    r = lambda *s, std=0.02: (torch.randn(*s, generator=g) * std)  # noqa: E731
    p = {}
    for blk in ("self_attn", "cross_attn"):
        for nm in ("q", "k", "v", "o"):
            p[f"{blk}.{nm}.weight"] = r(C, C).to(bf)
            p[f"{blk}.{nm}.bias"] = r(C).to(bf)
        p[f"{blk}.norm_q.weight"] = r(C).to(bf)
        p[f"{blk}.norm_k.weight"] = r(C).to(bf)
    p["norm3.weight"], p["norm3.bias"] = r(C), r(C)
    p["ffn.0.weight"], p["ffn.0.bias"] = r(F, C).to(bf), r(F).to(bf)
    p["ffn.2.weight"], p["ffn.2.bias"] = r(C, F).to(bf), r(C).to(bf)
    p["modulation"] = r(1, 6, C, std=0.1)
    x = r(rows_sample, C, std=1.0)
    e0 = r(6, C, std=0.1)
    k_lead = [r(chunk, H, 128, std=1.0).to(bf) for _ in range(c["n_lead"])]
    v_lead = [r(chunk, H, 128, std=1.0).to(bf) for _ in range(c["n_lead"])]
    ctx_k, ctx_v = r(TEXT_LEN, H, 128, std=1.0).to(bf), r(TEXT_LEN, H, 128, std=1.0).to(bf)
    cos, sin = ob.rope_grid(ob.rope_freqs(), c["grid"], c["start_frame"])
    # the reference's RoPE arithmetic for a chunk of this size (bf16 from 4,096 tokens, model_fast.py:1144-1148)
    rope_dt = torch.bfloat16 if f * gh * gw >= 4096 else torch.float32
    film = (r(rows_sample, C, std=0.1).to(bf), r(rows_sample, C, std=0.1).to(bf))
    # the chunk's own K/V are computed from the sample rows; the rest of the destination chunk is cached data
    k_lead = k_lead + [r(chunk - rows_sample, H, 128, std=1.0).to(bf)]
    v_lead = v_lead + [r(chunk - rows_sample, H, 128, std=1.0).to(bf)]
    t0 = time.perf_counter()
    for _ in range(blocks):
        ob.block_forward(p, x, e0, k_lead, v_lead, ctx_k, ctx_v, cos[:rows_sample], sin[:rows_sample], film=film,
                         mx=mx, rope_dtype=rope_dt)
    return time.perf_counter() - t0


def cpu_info():
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return os.cpu_count() or 1, model


def parity_rows(chunk, world, rank_rows, seed=5, n_random=24):
    """Query rows the parity check compares: on rank 0's shard the first and last rows, the rows on both sides
    of the 256-row CTA and 128-row tile boundaries, the ragged last query tile, and seeded random rows; on every
    other rank's shard a few rows (their K/V only, which rank 0 holds after the exchange)."""
    own = {0, 1, 127, 128, 255, 256, rank_rows - 1, rank_rows - 2}
    last_tile = (rank_rows - 1) // 128 * 128
    own |= {last_tile, last_tile + 1, max(last_tile - 1, 0)}
    g = torch.Generator().manual_seed(seed)
    own |= set(torch.randint(0, rank_rows, (n_random,), generator=g).tolist())
    own = sorted(r for r in own if 0 <= r < rank_rows)
    others = []
    for r in range(1, world):
        base = r * rank_rows
        others += [base, base + rank_rows // 2, base + rank_rows - 1]
    return own, others


def block_parity(stack, args, c, dims, dev, world, rank, L_loc, ks0, vs0, ctx, cache0, e0, freqs):
    """Checks block 0 of the timed stack against the CPU oracle (oracle/block.py, pinned to the reference's
    own block) on a sample of query rows: its output rows on rank 0, and the destination chunk's K and V rows of
    every rank (gathered into rank 0's cache under sequence parallelism). The oracle's window is the cached
    chunks plus the destination chunk as the GPU wrote it, with the sampled rows' K/V recomputed by the oracle
    (attention has no token mask, so the key order does not matter). Tolerances: rel-L2 <= 1e-2 on the block
    output (max-abs <= 0.15: the stack's FFN is MXFP8), rel-L2 <= 2e-2 on its update x_out - x, 1e-2 on K and V."""
    import lbw_b200._lib as L
    import lbw_b200.model as M
    from oracle import block as ob
    C, F, H = dims
    chunk = L_loc * world
    bf = torch.bfloat16
    # block 0's weights again: the timed stack drew them first from the same seed
    ref = M.BlockStack.synthetic(1, C, F, H, dev, seed=0, ffn_mx=True, lin_mx=args.lin_mx, free_sources=False)
    b0, r0 = stack.blocks[0], ref.blocks[0]
    same = all(torch.equal(a, b) if torch.is_tensor(a) else all(torch.equal(u, v) for u, v in zip(a, b))
               for a, b in ((b0._packed[k], r0._packed[k]) for k in b0._packed))
    p = {k: v.detach().cpu() for k, v in r0.state_dict().items() if not k.startswith("cam_")}
    del ref, r0
    gen = torch.Generator().manual_seed(1234)
    x_full = torch.randn(chunk, C, generator=gen).to(bf).float()
    fs_full = (torch.randn(chunk, C, generator=gen) * 0.1).to(bf)
    ft_full = (torch.randn(chunk, C, generator=gen) * 0.1).to(bf)
    a = rank * L_loc
    xs = x_full[a:a + L_loc].to(dev).contiguous()
    film = (fs_full[a:a + L_loc].to(dev).contiguous(), ft_full[a:a + L_loc].to(dev).contiguous())
    b0.forward_inplace(xs, e0, ks0, vs0, ctx, cache0, c["grid"], c["start_frame"], freqs, film=film, ws=stack._ws)
    torch.cuda.synchronize()
    L.check_device_status()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if rank != 0:
        return None
    own, others = parity_rows(chunk, world, L_loc)
    rows = own + others
    idx = torch.tensor(rows)
    k_dst = ks0[-1].view(chunk, H, 128).cpu()
    v_dst = vs0[-1].view(chunk, H, 128).cpu()
    keep = torch.ones(chunk, dtype=torch.bool)
    keep[idx] = False
    k_lead = [k.view(-1, H, 128).cpu() for k in ks0[:-1]] + [k_dst[keep]]
    v_lead = [v.view(-1, H, 128).cpu() for v in vs0[:-1]] + [v_dst[keep]]
    cos, sin = ob.rope_grid(ob.rope_freqs(), c["grid"], c["start_frame"])
    import lbw_b200.block as B
    names = [n for n in B.MX_LINEAR_NAMES] if args.lin_mx else ()
    ck, cv = ob.cross_kv(p, ctx.cpu(), mx_linears=names)
    t0 = time.perf_counter()
    import lbw_b200.rope as R
    r = ob.block_forward(p, x_full[idx], e0.cpu(), k_lead, v_lead, ck, cv, cos[idx], sin[idx],
                         film=(fs_full[idx], ft_full[idx]), mx=True, return_all=True, mx_linears=names,
                         rope_dtype=R.ROPE_DTYPE)
    t_oracle = time.perf_counter() - t0
    n = len(own)
    got = xs.cpu()[torch.tensor(own)]
    want, x_in = r["x"][:n], x_full[idx][:n]
    rel = lambda u, v: float((u.float() - v.float()).norm() / v.float().norm().clamp_min(1e-30))  # noqa: E731
    res = {"block": 0, "rows_checked": n, "kv_rows_checked": len(rows), "ranks_checked": world,
           "rel_l2": rel(got, want), "max_abs": float((got - want).abs().max()),
           "update_rel_l2": rel(got - x_in, want - x_in),
           "k_rel_l2": rel(k_dst[idx], r["k"]), "v_rel_l2": rel(v_dst[idx], r["v"]),
           "cross_k_rel_l2": rel(cache0["k"].view(-1, H, 128).cpu(), ck),
           "weights_match_timed_stack": bool(same), "oracle_s": round(t_oracle, 2),
           "oracle": "oracle/block.py (CPU restatement pinned to the reference block; MXFP8 FFN as OCP MX QDQ)",
           # max-abs 5e-2 is the bar of the bf16 block output; through the MXFP8 FFN a ~1e-4 difference upstream
           # moves single outputs by a few hundredths, so the MX block is held to rel-L2 and max-abs <= 0.15
           "tolerance": {"rel_l2": 1e-2, "max_abs": 0.15, "update_rel_l2": 2e-2, "kv_rel_l2": 1e-2}}
    res["ok"] = bool(same and res["rel_l2"] <= 1e-2 and res["max_abs"] <= 0.15 and res["update_rel_l2"] <= 2e-2
                     and res["k_rel_l2"] <= 1e-2 and res["v_rel_l2"] <= 1e-2 and res["cross_k_rel_l2"] <= 1e-2)
    return res


def run_reference(args):
    """--impl reference: the reference path's CPU implementation (the oracle port, oracle/block.py) on the
    host cores, rank 0 only, each step one block over a bounded sample of the chunk's query rows."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    c = CONFIGS[args.config]
    f, gh, gw = c["grid"]
    chunk = f * gh * gw
    layers = c["layers"]
    threads, model = cpu_info()
    # Warm-up on a small sample (thread pools, allocator), which also calibrates the per-row cost so that
    # the timed steps together stay near LBW_CPU_BUDGET_S seconds (default 150) whatever --steps is.
    probe_rows = 128
    t_probe = min(cpu_oracle_step(args.config, probe_rows, threads) for _ in range(max(1, min(args.warmup, 2))))
    budget = float(os.environ.get("LBW_CPU_BUDGET_S", "150"))
    rows = int(budget / max(args.steps, 1) / max(t_probe / probe_rows, 1e-9))
    rows = max(probe_rows, min(args.cpu_rows, rows // 8 * 8))
    times = [cpu_oracle_step(args.config, rows, threads) for _ in range(args.steps)]
    t_sample = statistics.median(times)                 # one timed step: 1 block over `rows` query rows
    t_full = t_sample * (chunk / rows) * layers         # the whole chunk through all blocks (extrapolated)
    value = chunk / t_full
    sample = (f"{rows} of {chunk} query rows through 1 of {layers} blocks (bf16 FFN) against the full "
              f"{(c['n_lead'] + 1) * chunk}-key window; CPU: {model}")
    out = {"metric": "chunk-forward tokens/s", "value": value, "unit": "tokens/s", "impl": "reference",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           # a timed step is the bounded sample below; the whole chunk forward is extrapolated from it
           "ms_per_step": t_sample * 1e3, "ms_per_step_kind": "measured sample (1 block, sample_rows rows)",
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "bf16 weights, fp32 residual and softmax (CPU torch)", "data": "synthetic",
           "config": config_of(args, world),
           "extrapolation": {"sample_rows": rows, "chunk_rows": chunk, "sample_blocks": 1, "blocks": layers,
                             "ms_sample_step": t_sample * 1e3, "ms_chunk_forward_extrapolated": t_full * 1e3,
                             "factor": (chunk / rows) * layers},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))
    return 0


def run_sweep(args):
    """Benchmark configuration c5: kernel sweep on one GPU. Chunk attention with 40 heads x 128 over
    Lq in {1560, 4680, 10800} x Lkv in {4096, 16384, 32768, 75600, 131072}; block-scaled FFN GEMMs (MXFP8 E4M3
    and E5M2, MXFP4 E2M1, E8M0 per 32) M in {4680, 10800, 43200} for up (K 5120 -> N 13824) and down
    (13824 -> 5120). One JSON line per
    point: TFLOP/s from CUDA events around each launch (median of 5, an L2 flush before each launch) and the
    fraction of the measured bf16 peak (burst: each kernel is timed alone)."""
    import __graft_entry__
    __graft_entry__.build()
    import lbw_b200.kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk, src = peaks()
    peak = pk["bf16_tflops"]
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16

    def timed(fn, reps=5):
        ts = []
        for _ in range(reps + 1):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts[1:])

    H, C = 40, 5120
    only = args.sweep_only
    # attn_c4: the headline step's self-attention launch alone (10,800 queries, 7 chunks of 10,800 keys), for
    # profiling one launch
    att = {"all": (1560, 4680, 10800), "attention": (1560, 4680, 10800), "attn_c4": (10800,)}.get(only, ())
    for lq in att:
        q = torch.randn(lq, C, generator=g, device=dev, dtype=bf)
        out = torch.empty(lq, C, dtype=bf, device=dev)
        for lkv in ((75600,) if only == "attn_c4" else (4096, 16384, 32768, 75600, 131072)):
            n_chunks = 7 if only == "attn_c4" else max(1, -(-lkv // 18900))
            rows = [lkv // n_chunks + (1 if i < lkv % n_chunks else 0) for i in range(n_chunks)]
            ks = [torch.randn(r, C, generator=g, device=dev, dtype=bf) for r in rows]
            vs = [torch.randn(r, C, generator=g, device=dev, dtype=bf) for r in rows]
            # the block's schedule: whole windows in full waves, the last partial wave cut into key ranges + merge
            n_tail, pieces = K.attention_tail_plan(lq, H, rows, dev)
            parts = K.attention_tail_workspace(lq, H, rows, dev)

            def run():
                K.chunk_attention_tail(q, ks, vs, parts, out=out)
            ms = timed(run)
            tf = 4.0 * lq * lkv * C / (ms / 1e3) / 1e12
            print(json.dumps({"sweep": "chunk_attention", "q_rows": lq, "kv_rows": lkv, "heads": H,
                              "cut_windows": n_tail, "pieces": pieces, "ms": ms, "tflops": tf,
                              "frac_of_peak": tf / peak, "peak": f"{src} bf16_tflops {peak}"}))
            del ks, vs, parts
    # block-scaled FFN GEMMs: MXFP8 E4M3 (the reference's default), E5M2 (its LINGBOT_MX_FP8 option) and MXFP4 E2M1;
    # the nominal dense rates are 2x (FP8) and 4x (FP4) the bf16 rate, so each point is also given against 2x / 4x
    # the measured bf16 peak
    fmts = {"mxfp8": ("e4m3", "e5m2", "e2m1"), "mxfp4": ("e2m1",), "all": ("e4m3", "e5m2", "e2m1")}.get(only, ())
    for fmt in fmts:
        mult = 4 if fmt == "e2m1" else 2
        for m in (4680, 10800, 43200):
            for kk, nn in ((5120, 13824), (13824, 5120)):
                a = torch.randn(m, kk, generator=g, device=dev, dtype=bf)
                w = (torch.randn(nn, kk, generator=g, device=dev) * 0.02).to(bf)
                ad, as_, _ = K.mx_quantize(a, fmt=fmt)
                wd, ws, _ = K.mx_quantize(w, fmt=fmt)
                o = torch.empty(m, nn, dtype=bf, device=dev)
                ms = timed(lambda: K.mx_linear(ad, as_, wd, ws, None, o, fmt=fmt))
                tf = 2.0 * m * kk * nn / (ms / 1e3) / 1e12
                print(json.dumps({"sweep": "mx_gemm", "format": fmt, "m": m, "k": kk, "n": nn, "ms": ms, "tflops": tf,
                                  "frac_of_bf16_peak": tf / peak, f"frac_of_{mult}x_bf16_peak": tf / (mult * peak),
                                  "peak": f"{src} bf16_tflops {peak}"}))
                del a, w, ad, as_, wd, ws, o
    # the block's bf16 GEMMs (q|k|v with the row sums of squares; o-projection with the gated residual + FiLM) at
    # the 1- and 8-GPU row counts of c4; 3 untimed launches first (an ncu capture can skip them with -s)
    for m in ((10800, 1350) if only in ("all", "gemm") else ()):
        h = torch.randn(m, C, generator=g, device=dev, dtype=bf)
        wqkv = (torch.randn(3 * C, C, generator=g, device=dev) * 0.02).to(bf)
        bqkv = (torch.randn(3 * C, generator=g, device=dev) * 0.02).to(bf)
        wo = (torch.randn(C, C, generator=g, device=dev) * 0.02).to(bf)
        bo = (torch.randn(C, generator=g, device=dev) * 0.02).to(bf)
        qr, kr, vv = (torch.empty(m, C, dtype=bf, device=dev) for _ in range(3))
        ss = torch.zeros(2, m, device=dev)
        xres = torch.randn(m, C, generator=g, device=dev)
        gate = torch.randn(C, generator=g, device=dev) * 0.1
        fs, ft = ((torch.randn(m, C, generator=g, device=dev) * 0.1).to(bf) for _ in range(2))
        for name, n, fn in (("qkv_rowss", 3 * C, lambda: K.qkv_proj(h, wqkv, bqkv, qr, kr, ss[0], ss[1], vv)),
                            ("o_proj_residual_film", C,
                             lambda: K.linear_residual(h, wo, bo, xres, gate=gate, film_scale=fs, film_shift=ft))):
            for _ in range(3):
                fn()
            ms = timed(fn, reps=3)
            tf = 2.0 * m * C * n / (ms / 1e3) / 1e12
            print(json.dumps({"sweep": "bf16_gemm", "name": name, "m": m, "k": C, "n": n, "ms": ms, "tflops": tf,
                              "frac_of_peak": tf / peak, "peak": f"{src} bf16_tflops {peak}"}))
    # the same Linears in MXFP8 (--lin-mx): activation quantiser, q|k|v, o-projection (+ gate + FiLM), cross-o
    for m in ((10800, 1350) if only in ("all", "linmx") else ()):
        h = torch.randn(m, C, generator=g, device=dev, dtype=bf)
        hq, hs = K.mx_buffers(m, C, dev)
        wqkv, wqkv_s, _ = K.mx_quantize((torch.randn(3 * C, C, generator=g, device=dev) * 0.02).to(bf))
        bqkv = (torch.randn(3 * C, generator=g, device=dev) * 0.02).to(bf)
        wo, wo_s, _ = K.mx_quantize((torch.randn(C, C, generator=g, device=dev) * 0.02).to(bf))
        bo = (torch.randn(C, generator=g, device=dev) * 0.02).to(bf)
        qr, kr, vv = (torch.empty(m, C, dtype=bf, device=dev) for _ in range(3))
        ss = torch.zeros(2, m, device=dev)
        xres = torch.randn(m, C, generator=g, device=dev)
        gate = torch.randn(C, generator=g, device=dev) * 0.1
        fs, ft = ((torch.randn(m, C, generator=g, device=dev) * 0.1).to(bf) for _ in range(2))
        K.mx_quantize(h, data=hq, scales=hs)
        F_ = 13824   # the MXFP8 FFN-down GEMM of the headline step (K = 13,824), for comparison
        uq, us, _ = K.mx_quantize(torch.randn(m, F_, generator=g, device=dev, dtype=bf))
        w2, w2_s, _ = K.mx_quantize((torch.randn(C, F_, generator=g, device=dev) * 0.02).to(bf))
        for name, n, fn in (("mx_quantize", 0, lambda: K.mx_quantize(h, data=hq, scales=hs)),
                            ("mx_qkv_rowss", 3 * C,
                             lambda: K.mx_qkv_proj(hq, hs, wqkv, wqkv_s, bqkv, qr, kr, ss[0], ss[1], vv)),
                            ("mx_o_proj_residual_film", C,
                             lambda: K.mx_linear_residual(hq, hs, wo, wo_s, bo, xres, gate=gate, film_scale=fs,
                                                          film_shift=ft)),
                            ("mx_cross_o_residual", C, lambda: K.mx_linear_residual(hq, hs, wo, wo_s, bo, xres)),
                            ("mx_ffn_down_residual", C,
                             lambda: K.mx_linear_residual(uq, us, w2, w2_s, bo, xres, gate=gate))):
            for _ in range(3):
                fn()
            ms = timed(fn, reps=3)
            kk = F_ if name == "mx_ffn_down_residual" else C
            rec = {"sweep": "lin_mx", "name": name, "m": m, "k": kk, "n": n, "ms": ms}
            if n:
                tf = 2.0 * m * kk * n / (ms / 1e3) / 1e12
                rec.update(tflops=tf, frac_of_2x_bf16_peak=tf / (2 * peak), peak=f"{src} bf16_tflops {peak}")
            else:
                rec.update(gbs=(m * C * 2 + m * C + m * C // 32) / (ms / 1e3) / 1e9)
            print(json.dumps(rec))
    # tile width at the per-rank row counts of 8 / 4 / 1 GPUs: automatic choice vs forced 128 / 256 (LBW_GEMM_TILE_N)
    for m in ((1350, 2700, 10800) if only == "tiles" else ()):
        F_ = 13824
        h = torch.randn(m, C, generator=g, device=dev, dtype=bf)
        hq, hs, _ = K.mx_quantize(h)
        wqkv = (torch.randn(3 * C, C, generator=g, device=dev) * 0.02).to(bf)
        bqkv = (torch.randn(3 * C, generator=g, device=dev) * 0.02).to(bf)
        wo = (torch.randn(C, C, generator=g, device=dev) * 0.02).to(bf)
        bo = (torch.randn(C, generator=g, device=dev) * 0.02).to(bf)
        w1, w1_s, _ = K.mx_quantize((torch.randn(F_, C, generator=g, device=dev) * 0.02).to(bf))
        b1 = (torch.randn(F_, generator=g, device=dev) * 0.02).to(bf)
        w2, w2_s, _ = K.mx_quantize((torch.randn(C, F_, generator=g, device=dev) * 0.02).to(bf))
        uq, us = K.mx_buffers(m, F_, dev)
        qr, kr, vv = (torch.empty(m, C, dtype=bf, device=dev) for _ in range(3))
        ss = torch.zeros(2, m, device=dev)
        xres = torch.randn(m, C, generator=g, device=dev)
        gate = torch.randn(C, generator=g, device=dev) * 0.1
        fs, ft = ((torch.randn(m, C, generator=g, device=dev) * 0.1).to(bf) for _ in range(2))
        ops = (("qkv_rowss", 5120, 3 * C, lambda: K.qkv_proj(h, wqkv, bqkv, qr, kr, ss[0], ss[1], vv)),
               ("o_proj_residual_film", 5120, C,
                lambda: K.linear_residual(h, wo, bo, xres, gate=gate, film_scale=fs, film_shift=ft)),
               ("cross_q_rowss", 5120, C, lambda: K.linear_rowss(h, wo, bo, qr, ss[0])),
               ("mx_ffn_up_gelu", 5120, F_, lambda: K.mx_linear_gelu(hq, hs, w1, w1_s, b1, uq, us)),
               ("mx_ffn_down_residual", F_, C, lambda: K.mx_linear_residual(uq, us, w2, w2_s, bo, xres, gate=gate)))
        for name, kk, n, fn in ops:
            rec = {"sweep": "tile_width", "name": name, "m": m, "k": kk, "n": n}
            for tn in ("auto", "128", "256"):
                if tn == "auto":
                    os.environ.pop("LBW_GEMM_TILE_N", None)
                else:
                    os.environ["LBW_GEMM_TILE_N"] = tn
                for _ in range(2):
                    fn()
                rec[f"ms_{tn}"] = timed(fn, reps=5)
            os.environ.pop("LBW_GEMM_TILE_N", None)
            print(json.dumps(rec))
    # KV splits and tail pieces of the self-attention at the per-rank query rows of 8 / 4 GPUs (c4 window: 7 chunks x
    # 10,800 keys)
    for lq in ((1350, 2700) if only == "tiles" else ()):
        q = torch.randn(lq, C, generator=g, device=dev, dtype=bf)
        out = torch.empty(lq, C, dtype=bf, device=dev)
        ks = [torch.randn(10800, C, generator=g, device=dev, dtype=bf) for _ in range(7)]
        vs = [torch.randn(10800, C, generator=g, device=dev, dtype=bf) for _ in range(7)]
        rec = {"sweep": "kv_splits", "q_rows": lq, "kv_rows": 75600,
               "auto": K.pick_kv_splits(lq, H, K.n_kv_tiles([10800] * 7))}
        for sp_ in range(1, 9):
            parts = K.attention_workspace(sp_, lq, H, dev) if sp_ > 1 else None

            def run():
                if parts is None:
                    K.chunk_attention(q, ks, vs, out=out)
                else:
                    K.chunk_attention_partial(q, ks, vs, sp_, *parts)
                    K.attention_merge(*parts, sp_, out)
            run()
            rec[f"ms_s{sp_}"] = timed(run, reps=3)
        # the block's tail schedule: the last partial wave of windows cut into `pieces` key ranges (0: planned)
        rec["tail_plan"] = K.attention_tail_plan(lq, H, [10800] * 7, dev)
        for pc in (0, 1, 2, 3, 4, 6, 8):
            parts = K.attention_tail_workspace(lq, H, [10800] * 7, dev, pc)

            def run_tail():
                K.chunk_attention_tail(q, ks, vs, parts, out=out, pieces=pc)
            run_tail()
            rec[f"ms_tail{pc}"] = timed(run_tail, reps=3)
        print(json.dumps(rec))
        del ks, vs
    return 0


def vae_flops(layout, h, w, t_steady=True):
    """Algorithmic FLOPs of one Decoder3d pass on a latent frame of h x w (real channels): every convolution
    2 * voxels * c_out * c_in * taps, the mid-block attention 4 * (hw)^2 * c plus its 1x1 projections."""
    t, total = 1, 0.0
    for kind, name, ci, co in layout:
        vox = t * h * w
        if kind == "conv":
            total += 2.0 * vox * co * ci * 27
        elif kind == "res":
            total += 2.0 * vox * co * ci * 27 + 2.0 * vox * co * co * 27 + (2.0 * vox * co * ci if ci != co else 0)
        elif kind == "attn":
            total += 4.0 * (h * w) ** 2 * ci * t + 2.0 * vox * ci * 4 * ci
        elif kind in ("up3d", "up2d"):
            if kind == "up3d" and t_steady:
                total += 2.0 * vox * 2 * ci * ci * 3
                t *= 2
            h, w = 2 * h, 2 * w
            total += 2.0 * t * h * w * co * ci * 9
        else:
            total += 2.0 * vox * 3 * ci * 27
    return total


def run_vae(args):
    """The Wan 2.1 VAE decode of 720p causal chunks (3 latent frames of 90 x 160 -> 12 frames of 720 x 1280 in
    the steady state) with the production decoder (dim 96) and seeded random weights; one step = one
    decode_chunk continuing the causal cache."""
    import __graft_entry__
    __graft_entry__.build()
    import lbw_b200.vae as V
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = V.WanVAEDecoder(dim=96).to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.no_grad():
        for name, prm in m.named_parameters():
            if name.endswith("gamma"):
                prm.copy_(1 + 0.1 * torch.randn(prm.shape, generator=g, device=dev))
            elif name.endswith("bias"):
                prm.copy_(0.02 * torch.randn(prm.shape, generator=g, device=dev))
            else:
                prm.copy_(torch.randn(prm.shape, generator=g, device=dev) / math.sqrt(prm[0].numel()))
    m.prepare()
    lat_t, lat_h, lat_w = 3, 90, 160
    z = torch.randn(16, lat_t, lat_h, lat_w, generator=g, device=dev)
    m.decode_chunk(z, first=True)                      # the video's first chunk (its first frame is not upsampled)
    for _ in range(args.warmup):
        m.decode_chunk(z)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            out = m.decode_chunk(z)
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    frames = out.shape[1]
    assert torch.isfinite(out).all()
    flops = vae_flops(m.layout, lat_h, lat_w) * lat_t
    pk, src = peaks()
    peak = pk.get("bf16_tflops_sustained") or pk["bf16_tflops"]
    tf = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "VAE decode frames/s (720p)", "value": frames / (ms / 1e3), "unit": "frames/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "bf16 (fp32 accumulation)", "data": "synthetic (seeded N(0,1) latent, random init)",
        "config": {"workload": "vae_decode_720p_chunk", "latent": [16, lat_t, lat_h, lat_w], "frames_out": frames,
                   "dim": 96, "l2": "activations and per-layer caches >> 126 MB"},
        "roofline": {"bound": "tensor", "kernel": "gemm_bf16_kernel<EpiConv> (implicit-GEMM conv)", "achieved": tf,
                     "peak": peak, "unit": "TFLOP/s", "frac": tf / peak, "flops_per_step": flops,
                     "peak_source": f"{src} bf16_tflops_sustained", "traffic": None},
        "clocks": clk.summary()}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="lbw", choices=["lbw", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=int(os.environ.get("LBW_CPU_ROWS", "1350")))
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle check of the first block on a row sample (run after the timed steps)")
    ap.add_argument("--sweep", action="store_true", help="kernel sweep (benchmark configuration c5) instead of the step")
    ap.add_argument("--sweep-only", default="all",
                    choices=["all", "attention", "attn_c4", "mxfp8", "mxfp4", "gemm", "linmx", "tiles"],
                    help="with --sweep: one family of points (gemm = the block's bf16 GEMMs at 10,800 and 1,350 rows)")
    ap.add_argument("--lin-mx", action="store_true",
                    help="every block Linear in MXFP8 (the reference's LINGBOT_LIN_MX option; not the headline config)")
    ap.add_argument("--vae", action="store_true",
                    help="the Wan 2.1 VAE decode of 720p chunks instead of the DiT step (one JSON line of its own)")
    ap.add_argument("--breakdown", action="store_true",
                    help="after the timed steps, time each phase of the block with CUDA event marks")
    args = ap.parse_args()
    if args.sweep:
        return run_sweep(args)
    if args.vae:
        return run_vae(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.build()
    import lbw_b200._lib as L
    import lbw_b200.block as B
    import lbw_b200.model as M
    import lbw_b200.rope as R
    import lbw_b200.sp as sp

    # the reference's RoPE arithmetic for this chunk: its model forward switches to bf16 RoPE for chunks of 4,096 or
    # more tokens (model_fast.py:1144-1148); the stack here is driven without the model, so set it the same way
    R.set_bf16_rope_for_forward(CONFIGS[args.config]["grid"][0] * CONFIGS[args.config]["grid"][1]
                                * CONFIGS[args.config]["grid"][2])
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        sp.set_group(None)

    c = CONFIGS[args.config]
    m = M.CONFIGS[c["model"]]
    C, H, F = m["dim"], m["num_heads"], m["ffn_dim"]
    layers = c["layers"]
    f, gh, gw = c["grid"]
    chunk = f * gh * gw
    if chunk % world:
        raise SystemExit(f"{chunk} query tokens do not split over {world} ranks")
    L_loc = chunk // world
    n_chunks = c["n_lead"] + 1
    lkv = n_chunks * chunk

    stack = M.BlockStack.synthetic(layers, C, F, H, dev, seed=0, ffn_mx=True, lin_mx=args.lin_mx)
    # the cached chunks and the text context are replicated: the same draws on every rank
    gk = torch.Generator(device=dev).manual_seed(1)
    bf = torch.bfloat16
    ks = [[torch.randn(1, chunk, H, 128, generator=gk, device=dev, dtype=bf) for _ in range(n_chunks)]
          for _ in range(layers)]
    vs = [[torch.randn(1, chunk, H, 128, generator=gk, device=dev, dtype=bf) for _ in range(n_chunks)]
          for _ in range(layers)]
    ctx = torch.randn(TEXT_LEN, C, generator=gk, device=dev, dtype=bf)
    e0 = torch.randn(6, C, generator=gk, device=dev) * 0.1      # the step's time embedding: the same on every rank
    g = torch.Generator(device=dev).manual_seed(2 + rank)
    caches = [{"k": torch.empty(TEXT_LEN, H, 128, dtype=bf, device=dev),
               "v": torch.empty(TEXT_LEN, H, 128, dtype=bf, device=dev)} for _ in range(layers)]
    films = [((torch.randn(L_loc, C, generator=g, device=dev) * 0.1).to(bf),
              (torch.randn(L_loc, C, generator=g, device=dev) * 0.1).to(bf)) for _ in range(layers)]
    x0 = torch.randn(L_loc, C, generator=g, device=dev).to(bf).float()
    xf = x0.clone()
    freqs = R.rope_freqs()
    # cross K/V of the text context: filled once per generation (not part of a denoising step)
    xf.copy_(x0)
    stack.forward_chunk(xf, e0, (ks, vs), ctx, caches, c["grid"], c["start_frame"], freqs, films=films,
                        fill_cross=True)
    torch.cuda.synchronize()
    L.check_device_status()

    def step(ev=None, phases=None, x=None):
        stack.forward_chunk(xf if x is None else x, e0, (ks, vs), ctx, caches, c["grid"], c["start_frame"], freqs,
                            films=films, attn_events=ev, phases=phases)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        xf.copy_(x0)
        step()
    barrier()
    L.check_device_status()

    attn_ev = []
    calls0 = L.CALLS[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            step(attn_ev)
        end.record()
        barrier()
    launches = L.CALLS[0] - calls0
    ms = start.elapsed_time(end) / args.steps
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in attn_ev)
    L.check_device_status()
    t = torch.tensor([ms, attn_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, attn_ms = float(t[0]), float(t[1])

    # per-phase times (outside the timed region): event marks between the block's kernels, summed over the
    # blocks of a step and averaged over steps; max over ranks
    breakdown = None
    if args.breakdown:
        marks = []
        barrier()
        for _ in range(args.steps):
            step(phases=marks)
        barrier()
        acc = {}
        prev = None
        for name, ev in marks:
            if name != "start" and prev is not None:
                acc[name] = acc.get(name, 0.0) + prev.elapsed_time(ev)
            prev = ev
        names = list(acc)
        t = torch.tensor([acc[n] / args.steps for n in names], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        breakdown = {n: round(float(v), 3) for n, v in zip(names, t)}

    # End to end through host buffers, pipelined as a serving loop runs it: step i's input is copied in (pinned
    # host -> device, on a copy stream) while step i - 1 computes, and its result is copied out while step i + 1
    # computes (two residual buffers). Every step's copies are inside the timed region, which ends when the last
    # result has reached the host.
    e2e = None
    if not args.no_e2e:
        xh = x0.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        bufs = [xf, torch.empty_like(xf)]
        cs = torch.cuda.Stream(device=dev)
        main = torch.cuda.current_stream(dev)

        def run_e2e(n):
            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_step = [torch.cuda.Event() for _ in range(2)]
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(main)
            cs.wait_event(start)
            with torch.cuda.stream(cs):
                bufs[0].copy_(xh, non_blocking=True)
                ev_in[0].record(cs)
            for i in range(n):
                b = i & 1
                main.wait_event(ev_in[b])
                step(x=bufs[b])
                ev_step[b].record(main)
                with torch.cuda.stream(cs):
                    if i + 1 < n:   # after the previous read-back of that buffer, in copy-stream order
                        bufs[b ^ 1].copy_(xh, non_blocking=True)
                        ev_in[b ^ 1].record(cs)
                    cs.wait_event(ev_step[b])
                    yh.copy_(bufs[b], non_blocking=True)
            main.wait_stream(cs)
            end.record(main)
            return start, end

        run_e2e(2)
        barrier()
        s2, e2 = run_e2e(args.steps)
        barrier()
        ms_e2e = s2.elapsed_time(e2) / args.steps
        t = torch.tensor([ms_e2e], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t[0])
        nbytes = xh.numel() * xh.element_size() * world
        e2e = {"value": chunk / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
               "d2h_bytes_per_step": nbytes, "ms_per_step": ms_e2e,
               "pipeline": "copy stream: step i's input in during step i - 1, its result out during step i + 1"}
    assert torch.isfinite(yh if e2e else xf).all(), "non-finite block output"

    # Parity of the timed stack's first block against the CPU oracle on a row sample (outside the timed region)
    parity = None
    if not args.no_parity:
        parity = block_parity(stack, args, c, (C, F, H), dev, world, rank, L_loc, ks[0], vs[0], ctx, caches[0], e0,
                              freqs)
    exchange = None
    if world > 1:
        pkv = [p for p in sp._PEERS.values()]
        exchange = {"kind": "copy engines over CUDA IPC (stream memory operations), not NCCL", "world": world,
                    "peers_opened": [p.world - 1 for p in pkv], "exchanges_per_step": layers}

    # DRAM traffic of one attention launch: an ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of
    # the c4 self-attention alone, 10,800 queries x 75,600 keys, measured 2,237.4 MB. K/V (re-read from L2 by
    # the query blocks of a head) dominate it, so another window is scaled by its K/V bytes; at N>1 a rank's
    # launch has fewer query blocks per head and no capture of its own, so the field is null there.
    kv_bytes = 4.0 * lkv * C
    attn_traffic = ATTN_TRAFFIC_C4_BYTES * kv_bytes / ATTN_KV_BYTES_C4 if world == 1 else None
    pk, src = peaks()
    fb, fm = flops_per_block(chunk, lkv, C, F)
    flops = (fb + fm) * layers
    attn_flops = 4 * L_loc * lkv * C
    attn_tf = attn_flops / (attn_ms / 1e3) / 1e12
    peak_tc = pk.get("bf16_tflops_sustained") or pk["bf16_tflops"]
    result = {
        "metric": "chunk-forward tokens/s", "value": chunk / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": ("bf16 (attention) + mxfp8 e4m3/e8m0 (every Linear, LINGBOT_LIN_MX)" if args.lin_mx else
                  "bf16 (attention, projections) + mxfp8 e4m3/e8m0 (FFN)"),
        "data": "synthetic (seeded N(0,1) latents / KV, N(0,0.02) weights, random init)",
        "config": config_of(args, world),
        "latency_ms": ms,
        "tc_frac_of_peak": flops / (ms / 1e3) / (peak_tc * 1e12 * world),
        "roofline": {"bound": "tensor", "kernel": "chunk_attn_kernel", "achieved": attn_tf, "peak": peak_tc,
                     "unit": "TFLOP/s", "frac": attn_tf / peak_tc, "traffic": attn_traffic,
                     "traffic_source": "ncu dram bytes of one c4 launch, scaled by K/V bytes" if attn_traffic else None,
                     "algorithmic_bytes": 2.0 * L_loc * C * 2 + kv_bytes,
                     "peak_source": f"{src} bf16_tflops_sustained", "flops_per_launch": attn_flops,
                     "ms_per_launch": attn_ms},
        "gpu_launches": launches,
        "e2e": e2e,
        "parity": parity,
    }
    if exchange is not None:
        result["exchange"] = exchange
    if breakdown is not None:
        result["phases_ms_per_step"] = breakdown
    if rank == 0:
        result["clocks"] = clk.summary()
    if rank == 0 and world == 1 and not args.no_cpu:
        threads, model = cpu_info()
        rows = args.cpu_rows
        cpu_oracle_step(args.config, 128, threads)     # warm-up (thread pools, allocator)
        t_cpu = cpu_oracle_step(args.config, rows, threads)
        cpu_value = rows / (t_cpu * layers)
        result["cpu_baseline"] = {"value": cpu_value, "unit": "tokens/s", "cores": threads, "kind": "port",
                                  "sample": f"oracle block (oracle/block.py, bf16 FFN) on {rows} of {chunk} query "
                                            f"rows, 1 block x{layers} extrapolated, full {lkv}-key window; {model}",
                                  "sample_rows": rows, "extrapolation_factor": (chunk / rows) * layers}
    if rank == 0:
        print(json.dumps(result))
    if world > 1:
        sp.close_peers()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
