"""Benchmark of the CrossDiT attention hot path on B200 (libkd_attn).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kd|reference] [--config 1]

Workload (default): BASELINE config 1 -- full 5 s clip self-attention, B2 (CFG cond +
uncond) x 31,744 tokens (31x32x32 grid) x 32 heads x d128, RMS-normed Q/K with 3D RoPE
(theta 1e4, axes 32/48/48), bf16 operands, fp32 accumulation, scale 1/sqrt(128).

A step is one kd_attn_self_attention call on resident f32 Q/K/V projections
([4096, L, 2] ggml layout, 3 x 1.04 GB > L2): the fused RMSNorm+RoPE+cast prologue
for Q, K and V, then the tcgen05 flash-attention kernel.  value = dense-equivalent
TFLOP/s = 4*B*H*L^2*d / step time.  With --gpus N > 1 the 32 heads are sharded
over the ranks (8 heads x 4 GPUs, ...) and the step ends with kd_attn_allgather_heads
(one NCCL all-gather + permute) -- strong scaling of the same job.

e2e: the same job through the public host-buffer call kd_attn_self_attention_host from
pinned HOST buffers: each step uploads the f32 Q/K/V projections, computes and downloads
the output, head group by head group with copies overlapping compute.

--impl reference: the reference's CPU algorithm (the oracle restatement of ggml's
flash_attn_ext with the RMSNorm/RoPE prologue; ggml itself is not available here)
on this host's cores, timed on a bounded slice of the same workload and scaled.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kandinsky.cpp_b200"))

METRIC = "attn TFLOP/s (dense-equiv) at 31744 tok x 32h x d128"
UNIT = "TFLOP/s"

CONFIGS = {
    0: dict(name="cfg0 self-attn B1 L1280 (5x16x16) H32 d128, f32 Q / f16 K,V", N=1, grid=(5, 16, 16), H=32,
            op="f16", out="f32"),
    1: dict(name="cfg1 self-attn B2 L31744 (31x32x32) H32 d128 bf16", N=2, grid=(31, 32, 32), H=32, op="bf16",
            out="bf16"),
    2: dict(name="cfg2 cross-attn B2 Lq31744 (31x32x32) x Lk256 (valid U[40,256]) H32 d128 bf16", kind="cross",
            N=2, grid=(31, 32, 32), Lk=256, H=32, op="bf16", out="bf16"),
    3: dict(name="cfg3 self-attn B2 L71424 (31x48x48) H32 d128 bf16", N=2, grid=(31, 48, 48), H=32, op="bf16",
            out="bf16"),
    4: dict(name="cfg4 block-sparse self-attn B1 L62464 (61x32x32) H32 d128 bf16, 64x64 tiles", kind="sparse",
            N=1, grid=(61, 32, 32), H=32, op="bf16", out="bf16", p_random=0.14),
}


def block_sparse_tiles(grid, p_random, seed=4):
    """Kept 64x64 tiles of config 4 (numpy bool [nt, nt]): tile i = (frame i//16, strip i%16) of a
    32x32-token frame (1024 tokens = 16 tiles of 2 latent rows); kept = diagonal, |df| <= 1 and
    |ds| <= 1 (temporal window over spatially adjacent tiles), plus seeded random tiles at p_random."""
    import numpy as np
    nt_tok = grid[0] * grid[1] * grid[2]
    nt = nt_tok // 64
    per_frame = grid[1] * grid[2] // 64
    i = np.arange(nt)
    f, s = i // per_frame, i % per_frame
    keep = (np.abs(f[:, None] - f[None, :]) <= 1) & (np.abs(s[:, None] - s[None, :]) <= 1)
    keep |= np.eye(nt, dtype=bool)
    keep |= np.random.default_rng(seed).random((nt, nt)) < p_random
    return keep


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), "measured"
    return 1590.0, 1400.0, "fallback"


def profile_traffic():
    """dram bytes per FA launch from the committed ncu summary (None if absent)."""
    p = os.path.join(ROOT, "profiles", "fmha_fwd_bf16_cfg1.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of the job's GPUs, sampled every 100 ms while the timed
    region runs (entering waits for the first sample, so sampling is live when timing starts).  One
    process per node, started by local rank 0 for all of the node's GPUs: one poller per rank
    perturbed 8-GPU steps measurably."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = list(devices)   # nvidia-smi indices; empty = this rank does not sample
        self.proc = None
        self.lines = []

    def __enter__(self):
        if not self.devices:
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", ",".join(str(d) for d in self.devices),
                                          f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
                time.sleep(0.01)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        if not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def node_gpus(local, ws):
    """nvidia-smi indices of the GPUs this node's ranks use (rank i on cuda:i, through CUDA_VISIBLE_DEVICES)."""
    per_node = int(os.environ.get("LOCAL_WORLD_SIZE", str(ws)))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = [v.strip() for v in vis.split(",")] if vis else [str(i) for i in range(per_node)]
    return ids[:per_node]


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_model():
    """The host CPU's model name (first /proc/cpuinfo entry), or platform.processor()."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def sample_rows_for_cpu(L, budget_flop, d=128):
    """query rows of one (batch, head) pair so the CPU oracle does about budget_flop of work."""
    per_row = 4.0 * L * d
    return max(16, min(L, int(budget_flop / per_row)))


def cpu_reference(cfg, seconds_target=15.0, threads=None):
    """Time the CPU oracle (ggml-faithful flash_attn_ext + prologue) on a slice; returns a dict."""
    import numpy as np

    import oracle
    threads = threads or os.cpu_count() or 1
    os.environ["KD_ORACLE_THREADS"] = str(threads)
    nt, nh, nw = cfg["grid"]
    L = nt * nh * nw
    d = 128
    kv_type = oracle.F16 if cfg["op"] == "f16" else oracle.BF16
    # calibrate on a small slice, then size the sample for ~seconds_target
    q = oracle.philox_randn(11, L * d, 0).reshape(1, L, d)
    k = oracle.philox_randn(11, L * d, 1).reshape(1, L, d)
    v = oracle.philox_randn(11, L * d, 2).reshape(1, L, d)
    tab = oracle.visual_rope_table(cfg["grid"])

    def run(rows):
        t0 = time.perf_counter()
        qn = oracle.rope_apply(oracle.rms_norm_heads(q[:, :rows], d), 1, d, tab[:rows])
        kn = oracle.rope_apply(oracle.rms_norm_heads(k, d), 1, d, tab)
        k4 = oracle.to_type(kn[:, None], kv_type)
        v4 = oracle.to_type(v[:, None], kv_type)
        oracle.flash_attn_ext(qn[:, None], k4, v4, mode=oracle.GGML)
        return time.perf_counter() - t0

    # per-row cost from two small runs (each run also pays the fixed K-side prologue and casts)
    r_a, r_b = min(L, 64), min(L, 512)
    t_a, t_b = run(r_a), run(r_b)
    slope = max((t_b - t_a) / max(r_b - r_a, 1), 1e-6)
    rows = int(min(L, max(r_b, r_b + (seconds_target - t_b) / slope)))
    planes, t = 0, 0.0
    if rows < L:
        t, planes = run(rows), 1
        flop_sample = 4.0 * rows * L * d
        what = f"1 (batch, head) plane x {rows} of {L} query rows"
    else:  # a whole plane is quicker than the target: repeat whole planes (same work each)
        while planes == 0 or (t < seconds_target and planes < cfg["N"] * cfg["H"]):
            t += run(L)
            planes += 1
        flop_sample = planes * 4.0 * L * L * d
        what = f"{planes} whole (batch, head) planes of {cfg['N'] * cfg['H']}"
    full_flop = 4.0 * cfg["N"] * cfg["H"] * L * L * d
    ms_full = t * 1e3 * full_flop / flop_sample
    return {"value": flop_sample / t / 1e12, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model(),
            "sample": f"{what} (prologue + ggml-faithful flash_attn_ext), {t:.1f} s on {threads} threads; "
                      f"scaled by the FLOP ratio to {ms_full / 1e3:.0f} s per full call",
            "ms_per_call_scaled": ms_full}


def run_reference(args, cfg):
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    steps = []
    cb = None
    # each step is a bounded sample; the whole arm stays near 150 s of CPU time for any --steps
    per_step = max(2.0, min(args.ref_seconds, 150.0 / max(1, args.warmup + args.steps)))
    for i in range(args.warmup + args.steps):
        cb = cpu_reference(cfg, seconds_target=per_step)
        if i >= args.warmup:
            steps.append(cb)
    vals = [s["value"] for s in steps]
    val = sum(vals) / len(vals)
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": steps[-1]["ms_per_call_scaled"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": cfg["op"],
            "data": "synthetic (seeded Philox4x32-10 N(0,1), the reference's generator)",
            "config": {"workload": cfg["name"], "global_batch": cfg["N"], "seq_len": L_of(cfg), "heads": cfg["H"],
                       "head_dim": 128, "parallelism": "cpu", "l2": "n/a"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model")},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def L_of(cfg):
    nt, nh, nw = cfg["grid"]
    return nt * nh * nw


def _timed(torch, stream, fn, steps, warmup):
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def run_other(args, cfg, ctx, kd_attn, torch, q, k, v, rope, op, out_dt, stream):
    """Configs 2 (cross-attention, variable text length) and 4 (64x64 block-sparse self-attention)."""
    import numpy as np
    N, H, d, L = cfg["N"], cfg["H"], 128, L_of(cfg)
    dev = q.device
    opdt = torch.bfloat16 if op == kd_attn.BF16 else torch.float16
    pk, _, pk_kind = peaks()
    if cfg["kind"] == "cross":
        Lk = cfg["Lk"]
        kv_len = torch.from_numpy(np.random.default_rng(2).integers(40, Lk + 1, size=N).astype(np.int32)).to(dev)
        kt = torch.empty(N * Lk * H * d, device=dev)
        vt = torch.empty_like(kt)
        ctx.fill_randn(kt, seed=3, offset=1)
        ctx.fill_randn(vt, seed=3, offset=2)
        kt, vt = (kt * 0.5).view(N, Lk, H * d), (vt * 0.5).view(N, Lk, H * d)
        out = torch.empty(N, L, H * d, device=dev, dtype=out_dt)
        ms = _timed(torch, stream, lambda: ctx.cross_attention(q, kt, vt, H, out, kv_len=kv_len, op_type=op,
                                                                stream=stream), args.steps, args.warmup)
        qs = torch.empty(N, H, L, d, device=dev, dtype=opdt)
        ks = torch.empty(N, H, Lk, d, device=dev, dtype=opdt)
        vs = torch.empty_like(ks)
        ctx.qk_prologue(q, kt, vt, qs, ks, vs, stream=stream)
        o4 = out.view(N, L, H, d)
        fa_ms = _timed(torch, stream, lambda: ctx.flash_attn_ext(qs, ks, vs, o4, kv_len=kv_len, stream=stream),
                       args.steps, args.warmup)
        ctx.device_status()
        flop = 4.0 * N * H * L * Lk * d
        flop_valid = 4.0 * H * L * d * float(kv_len.sum().item())
        fa_bytes = (N * H * L * d * 2) * 2 + N * H * Lk * d * 2 * 2     # Q + O (bf16) + K + V
        call_bytes = N * L * H * d * 4 + 2 * N * Lk * H * d * 4 + N * H * (L + 2 * Lk) * d * 2 + fa_bytes
        return {"metric": "cross-attn TFLOP/s (dense-equiv) and HBM GB/s", "config": {"workload": cfg["name"],
                "kv_len": kv_len.tolist()}, "ms_per_step": ms, "value": flop / (ms * 1e-3) / 1e12, "unit": UNIT,
                "tflops_valid_keys": flop_valid / (ms * 1e-3) / 1e12,
                "call_gbs": call_bytes / (ms * 1e-3) / 1e9,
                "flash_kernel": {"ms": fa_ms, "gbs": fa_bytes / (fa_ms * 1e-3) / 1e9,
                                 "frac_of_hbm": fa_bytes / (fa_ms * 1e-3) / 1e9 / hbm_peak(),
                                 "algorithmic_bytes": fa_bytes}}
    # block-sparse
    keep = block_sparse_tiles(cfg["grid"], cfg["p_random"])
    nt = keep.shape[0]
    density = float(keep.mean())
    qt = keep.reshape(nt // 2, 2, nt // 2, 2).any(axis=(1, 3))              # 128-row x 128-key products computed
    bits = torch.from_numpy(kd_attn.tile_bitmap(keep)).to(dev)              # 976 x 122 B = 119 KB
    keep_t = torch.from_numpy(keep).to(dev)
    cond = keep_t.repeat_interleave(64, 0).repeat_interleave(64, 1)
    mask = torch.zeros(1, 1, L, L, device=dev, dtype=torch.float16)
    mask.view(L, L).masked_fill_(~cond, float("-inf"))
    del cond, keep_t
    qs = torch.empty(N, H, L, d, device=dev, dtype=opdt)
    ks, vs = torch.empty_like(qs), torch.empty_like(qs)
    out = torch.empty(N, L, H, d, device=dev, dtype=out_dt)

    # the step: fused prologue + flash with the 64x64 tile bitmap (the block mask in 119 KB)
    def step():
        ctx.qk_prologue(q, k, v, qs, ks, vs, rope=rope, stream=stream)
        ctx.flash_attn_ext(qs, ks, vs, out, tile_mask=bits, stream=stream)

    ms = _timed(torch, stream, step, args.steps, args.warmup)
    ctx.tile_stats(reset=True, stream=stream)
    fa_ms = _timed(torch, stream, lambda: ctx.flash_attn_ext(qs, ks, vs, out, tile_mask=bits, stream=stream),
                   args.steps, args.warmup)
    loaded, pairs = ctx.tile_stats(reset=True, stream=stream)
    launches = args.steps + max(args.warmup, 3)  # _timed's warm-up and timed calls
    # the same call from the dense f16 mask (7.8 GB, classified on the device every call)
    fa_dense_ms = _timed(torch, stream, lambda: ctx.flash_attn_ext(qs, ks, vs, out, mask=mask, stream=stream),
                         args.steps, args.warmup)
    ctx.device_status()
    dense = 4.0 * N * H * L * L * d
    actual = dense * density
    per_launch_pairs = pairs / launches
    return {"metric": "block-sparse attn TFLOP/s (dense-equiv and kept-tile)", "config": {"workload": cfg["name"],
            "tile_density": density, "computed_fraction_128x128": float(qt.mean()),
            "units": "head pairs (128 rows x 2 heads; every loaded K/V tile is used by both Q tiles)",
            "mask": "64x64 tile bitmap (kd_attn_flash_ext tile_mask)"},
            "ms_per_step": ms, "value": dense / (ms * 1e-3) / 1e12, "unit": UNIT,
            "tflops_kept_tiles": actual / (ms * 1e-3) / 1e12,
            "tile_counters": {"loaded_per_launch": loaded / launches, "expected_loaded": float(qt.sum()) * N * H,
                              "computed_per_launch": per_launch_pairs, "expected_computed": float(qt.sum()) * N * H},
            "flash_kernel_tile_mask": {"ms": fa_ms, "dense_equiv_tflops": dense / (fa_ms * 1e-3) / 1e12,
                                       "kept_tile_tflops": actual / (fa_ms * 1e-3) / 1e12,
                                       "tflops_on_computed_tiles": dense * float(qt.mean()) / (fa_ms * 1e-3) / 1e12,
                                       "peak": pk, "peak_kind": pk_kind},
            "flash_kernel_dense_mask_ms": fa_dense_ms}


def exchange_check(ctx, torch, dist, proj, out_full, rope, op, out_dt, ws, rank, N, L, Hs, Cs, dev, stream):
    """After the timed sharded steps, every rank's out_full must hold every rank's heads.  Each rank
    recomputes, with the single-GPU kd_attn_self_attention, its own heads and those of the next rank
    (from that rank's seed) and requires the columns of its out_full -- its own written locally,
    the peer's written over NVLink by the peer's flash kernel -- to be bit-identical.  The outcome
    is min-reduced over the ranks, so every rank reports the same one."""
    checked = []
    ok = True
    for owner in (rank, (rank + 1) % ws):
        ins = [proj(off, owner) for off in range(3)]
        ref = torch.empty(N, L, Cs, device=dev, dtype=out_dt)
        ctx.self_attention(*ins, Hs, ref, rope=rope, op_type=op, stream=stream)
        torch.cuda.synchronize()
        got = out_full[:, :, owner * Cs:(owner + 1) * Cs]
        same = bool(torch.equal(got, ref))
        ndiff = 0 if same else int((got != ref).sum().item())
        checked.append({"heads_of_rank": owner, "rows": N * L, "bit_identical": same, "elements_differing": ndiff})
        ok = ok and same
        del ins, ref
    flag = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return {"status": "pass" if int(flag.item()) == 1 else "fail", "ranks": ws, "rank0_checked": checked,
            "how": "each rank recomputes its own and the next rank's heads (kd_attn_self_attention, single GPU) "
                   "and compares them bit for bit with its out_full copy after the timed steps; min over ranks"}


def extra_measurements(args, ctx, kd_attn, torch, q, k, v, rope, dev, stream):
    """Single-GPU side measurements printed with the headline line.
    cfg2: the config-2 cross-attention call (the config-1 Q projections are config 2's Q: same shape,
          N(0,1)) and its flash kernel alone, in HBM GB/s.
    ggml_semantics: config 1 through kd_attn_flash_ext the way ops.hpp:176 feeds it -- f32 Q
          (rounded to f16 inside the call), f16 K/V, f32 output -- beside the same call with Q
          already f16, whose difference is the Q-rounding kernel's share."""
    res = {}
    cfg2 = dict(CONFIGS[2])
    if args.batch:  # profiling overrides shape config 1's Q, which config 2 reuses
        cfg2["N"] = args.batch
    if args.heads:
        cfg2["H"] = args.heads
    if args.frames:
        cfg2["grid"] = (args.frames,) + tuple(cfg2["grid"][1:])
    r2 = run_other(args, cfg2, ctx, kd_attn, torch, q, None, None, rope, kd_attn.BF16, torch.bfloat16, stream)
    res["cfg2"] = {"workload": cfg2["name"], "kv_len": r2["config"]["kv_len"], "call_ms": r2["ms_per_step"],
                   "flash_kernel_ms": r2["flash_kernel"]["ms"], "flash_kernel_gbs": r2["flash_kernel"]["gbs"],
                   "flash_kernel_frac_of_hbm": r2["flash_kernel"]["frac_of_hbm"],
                   "algorithmic_bytes": r2["flash_kernel"]["algorithmic_bytes"],
                   "bytes": "Q + O (bf16) + K + V of the valid-length-independent padded shape"}
    N, L, C = q.shape
    H, d = C // 128, 128
    qf = torch.empty(N, H, L, d, device=dev)
    q16 = torch.empty(N, H, L, d, device=dev, dtype=torch.float16)
    k16, v16 = torch.empty_like(q16), torch.empty_like(q16)
    ctx.qk_prologue(q, k, v, q16, k16, v16, rope=rope, stream=stream)
    ctx.prologue(q, H, qf, rope=rope, stream=stream)
    of = torch.empty(N, L, H, d, device=dev)
    ms_f32q = _timed(torch, stream, lambda: ctx.flash_attn_ext(qf, k16, v16, of, stream=stream), args.steps,
                     args.warmup)
    ms_f16q = _timed(torch, stream, lambda: ctx.flash_attn_ext(q16, k16, v16, of, stream=stream), args.steps,
                     args.warmup)
    ctx.device_status()
    flop = 4.0 * N * H * L * L * d
    res["ggml_semantics"] = {
        "call": "kd_attn_flash_ext, Q f32 [128, L, H, N], K/V f16, out f32 [128, H, L, N] (ops.hpp:176)",
        "ms": ms_f32q, "tflops": flop / (ms_f32q * 1e-3) / 1e12,
        "ms_q_already_f16": ms_f16q, "q_rounding_ms": ms_f32q - ms_f16q,
        "q_rounding_share": (ms_f32q - ms_f16q) / ms_f32q}
    del qf, q16, k16, v16, of
    res["lite_video"] = lite_video(args, ctx, kd_attn, torch, q, k, v, rope, dev, stream)
    res["projection_attention"] = projection_attention(args, ctx, kd_attn, torch, q, rope, dev, stream)
    return res


def lite_video(args, ctx, kd_attn, torch, q, k, v, rope, dev, stream):
    """The lite video model's self-attention (CrossDiTConfig::lite_video, crossdit.hpp:48-56: 28 heads of
    head_dim 64, RoPE axes {16, 24, 24}, scale {1, 2, 2}) over config 1's tokens: the first 1792 channels
    of config 1's projections, bf16 operands.  The whole call (prologue + flash) and the flash kernel
    alone, in dense-equivalent TFLOP/s (4 B H L^2 d)."""
    N, L, _ = q.shape
    H, d = 28, 64
    ql, kl, vl = (x[:, :, :H * d] for x in (q, k, v))          # strided views: rows of 4096 floats
    rope_l = kd_attn.Rope3D.make(tuple(rope.grid), axes=(16, 24, 24), scale=(1, 2, 2))
    out = torch.empty(N, L, H * d, device=dev, dtype=torch.bfloat16)
    call_ms = _timed(torch, stream, lambda: ctx.self_attention(ql, kl, vl, H, out, rope=rope_l, op_type=kd_attn.BF16,
                                                               stream=stream), args.steps, args.warmup)
    qs = torch.empty(N, H, L, d, device=dev, dtype=torch.bfloat16)
    ks, vs = torch.empty_like(qs), torch.empty_like(qs)
    ctx.qk_prologue(ql, kl, vl, qs, ks, vs, rope=rope_l, stream=stream)
    o4 = out.view(N, L, H, d)
    fa_ms = _timed(torch, stream, lambda: ctx.flash_attn_ext(qs, ks, vs, o4, stream=stream), args.steps, args.warmup)
    del qs, ks, vs
    # the whole module (DiTSelfAttention::forward of the lite model): q8_0 Q/K/V/out weights [1792, 1792]
    # with biases, the first 1792 channels of config 1's projections as the hidden states
    C = H * d
    ws = [_q8_0_weight(torch, C, C, 20 + i, dev) for i in range(4)]
    lin = [kd_attn.KdLinear.of(ws[i], kd_attn.Q8_0, C, C, torch.randn(C, device=dev) * 0.1) for i in range(4)]
    y = torch.empty(N, L, C, device=dev)
    block_ms = _timed(torch, stream, lambda: ctx.self_attention_block(ql, *lin, H, y, rope=rope_l, stream=stream),
                      args.steps, args.warmup)
    ctx.device_status()
    flop = 4.0 * N * H * L * L * d
    gemm_flop = 4 * 2.0 * N * L * C * C
    return {"workload": f"lite video self-attn B{N} L{L} H{H} d{d} bf16", "call_ms": call_ms,
            "call_tflops": flop / (call_ms * 1e-3) / 1e12, "flash_kernel_ms": fa_ms,
            "flash_kernel_tflops": flop / (fa_ms * 1e-3) / 1e12,
            "self_attention_block_ms": block_ms,
            "self_attention_block": "kd_attn_self_attention_block, n_head 28: x f32 [1792, L, N] -> q8_0 QKV "
                                    "projection -> flash -> q8_0 out-projection -> y f32",
            "self_attention_block_tflops": (flop + gemm_flop) / (block_ms * 1e-3) / 1e12}


def _q8_0_weight(torch, rows, cols, seed, dev):
    """Synthetic q8_0 Linear weight [cols, rows] (ggml ne): rows of 34-byte blocks, f16 scale 1/(127*64), int8
    values uniform in [-127, 127] -- a valid block stream of the converter's format."""
    g = torch.Generator(device=dev).manual_seed(seed)
    raw = torch.empty(rows, cols // 32, 34, dtype=torch.uint8, device=dev)
    qv = torch.randint(-127, 128, (rows, cols // 32, 32), device=dev, dtype=torch.int16, generator=g).to(torch.int8)
    raw[..., :2] = torch.full((rows, cols // 32, 1), 1.0 / (127 * 64), dtype=torch.float16,
                              device=dev).view(torch.uint8)
    raw[..., 2:] = qv.view(torch.uint8)
    return raw.view(rows, -1)


def projection_attention(args, ctx, kd_attn, torch, x, rope, dev, stream):
    """Config 1's self-attention block from the hidden states: to_query/to_key/to_value with q8_0 weights and
    f32 biases (crossdit.hpp:123-125) fused with RMSNorm + RoPE + cast (kd_attn_qkv_projection), then the flash
    kernel on its bf16 operands.  x is the config-1 synthetic N(0,1) tensor [4096, L, N].  A plain cuBLAS bf16
    GEMM of the same shape (bf16 out, no epilogue work) is timed beside it as the library reference."""
    N, L, K = x.shape
    H, d = K // 128, 128
    C = H * d
    ws = [_q8_0_weight(torch, C, K, 11 + i, dev) for i in range(3)]
    bias = [torch.randn(C, device=dev) * 0.1 for _ in range(3)]
    lin = [kd_attn.KdLinear.of(ws[i], kd_attn.Q8_0, K, C, bias[i]) for i in range(3)]
    outs = [torch.empty(N, H, L, d, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    o = torch.empty(N, L, H, d, device=dev, dtype=torch.bfloat16)
    proj = lambda: ctx.qkv_projection(x, *lin, *outs, rope=rope, stream=stream)
    attn = lambda: ctx.flash_attn_ext(*outs, o, stream=stream)
    ms_proj = _timed(torch, stream, proj, args.steps, args.warmup)
    ms_attn = _timed(torch, stream, attn, args.steps, args.warmup)
    ms_both = _timed(torch, stream, lambda: (proj(), attn()), args.steps, args.warmup)
    # the whole DiTSelfAttention::forward through one call: projection, attention, q8_0 out-projection
    wo = _q8_0_weight(torch, C, C, 14, dev)
    lin_o = kd_attn.KdLinear.of(wo, kd_attn.Q8_0, C, C, torch.randn(C, device=dev) * 0.1)
    y = torch.empty(N, L, C, device=dev)
    ms_block = _timed(torch, stream, lambda: ctx.self_attention_block(x, *lin, lin_o, C // 128, y, rope=rope,
                                                                      stream=stream), args.steps, args.warmup)
    ctx.device_status()
    del outs, o, ws, bias, lin, wo, lin_o, y
    xb = x.reshape(-1, K).to(torch.bfloat16)
    wb = torch.randn(3 * C, K, device=dev, dtype=torch.bfloat16)
    with torch.cuda.stream(stream):
        ms_lib = _timed(torch, stream, lambda: torch.matmul(xb, wb.t()), args.steps, args.warmup)
    del xb, wb
    pk, _, pk_kind = peaks()
    proj_flop = 2.0 * N * L * K * 3 * C
    attn_flop = 4.0 * N * H * L * L * d
    return {
        "workload": "config 1 block: x [4096, 31744, 2] f32 -> q8_0 QKV projection + bias + RMSNorm + RoPE -> "
                    "bf16 operands -> flash attention",
        "projection_ms": ms_proj, "projection_tflops": proj_flop / (ms_proj * 1e-3) / 1e12,
        "projection_frac_of_bf16_burst": proj_flop / (ms_proj * 1e-3) / 1e12 / pk, "peak_kind": pk_kind,
        "attention_ms": ms_attn, "block_ms": ms_both,
        "block_tflops": (proj_flop + attn_flop) / (ms_both * 1e-3) / 1e12,
        "f32_projection_bytes_avoided": 2 * 3 * N * L * C * 4,
        "self_attention_block_ms": ms_block,
        "self_attention_block": "kd_attn_self_attention_block: x f32 -> QKV projection -> flash -> q8_0 "
                                "out-projection -> y f32 [4096, L, N] (crossdit.hpp:117-154)",
        "self_attention_block_tflops": (proj_flop * 4 / 3 + attn_flop) / (ms_block * 1e-3) / 1e12,
        "library_gemm_ms": ms_lib,
        "library_gemm": "torch.matmul bf16 [2L, 4096] x [4096, 12288] (cuBLAS), bf16 out, no bias/norm/RoPE",
        "projection_call_includes": "q8_0 -> bf16 weight expansion, x f32 -> bf16, RoPE table, fused GEMM"}


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)).get("hbm_gbs", 6650.0)
    return 6650.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kd", choices=["kd", "reference"])
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--ref-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config-2 and ggml-semantics measurements of the single-GPU line")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (profiling runs)")
    ap.add_argument("--heads", type=int, default=None, help="override the config's head count (profiling runs)")
    ap.add_argument("--frames", type=int, default=None,
                    help="override the config's number of latent frames (grid[0]; profiling runs)")
    ap.add_argument("--fa-only", action="store_true",
                    help="time only the flash-attention kernel on prologue-made operands (profiling runs)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["N"] = args.batch
    if args.heads:
        cfg["H"] = args.heads
    if args.frames:
        cfg["grid"] = (args.frames,) + tuple(cfg["grid"][1:])
    if args.batch or args.heads or args.frames:
        cfg["name"] += f" [override B{cfg['N']} H{cfg['H']} grid {'x'.join(str(g) for g in cfg['grid'])}]"

    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist

    import kd_attn

    ws, rank, local = dist_setup()
    if ws != args.gpus:
        print(f"note: WORLD_SIZE={ws} but --gpus {args.gpus}; using WORLD_SIZE", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        # NCCL's init lines ("... nranks N ... Init COMPLETE") show every communicator's size; they go to
        # stderr so that stdout keeps the one JSON line
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() in ("", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
            os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", init_method="env://", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=120))
    N, H, d = cfg["N"], cfg["H"], 128
    L = L_of(cfg)
    assert H % ws == 0, "heads must divide over the ranks"
    Hs = H // ws
    Cs = Hs * d
    op = kd_attn.BF16 if cfg["op"] == "bf16" else kd_attn.F16
    out_dt = torch.bfloat16 if cfg["out"] == "bf16" else torch.float32

    nccl_id = None
    if ws > 1:
        obj = [kd_attn.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    ctx = kd_attn.Context(device=local, n_ranks=ws, rank=rank, nccl_id=nccl_id)
    stream = torch.cuda.current_stream()

    # inputs: this rank's column shard (heads [rank*Hs, (rank+1)*Hs)) of the Q/K/V projections
    def proj(offset, owner=rank):
        """rank `owner`'s column shard of one projection (seed 1 + owner)."""
        t = torch.empty(N, L, Cs, device=dev)
        full = torch.empty(N * L * Cs, device=dev)
        ctx.fill_randn(full, seed=1 + owner, offset=offset)
        t.copy_(full.view(N, L, Cs))
        return t

    q, k, v = proj(0), proj(1), proj(2)
    rope = kd_attn.Rope3D.make(cfg["grid"])
    out_shard = torch.empty(N, L, Cs, device=dev, dtype=out_dt)
    # N > 1: every rank's copy of the full output is mapped into every other rank; the flash epilogue
    # stores each row into all copies (kd_attn_self_attention_sharded)
    out_full = ctx.symmetric_tensor((N, L, H * d), out_dt) if ws > 1 else out_shard

    def step():
        if ws > 1:
            ctx.self_attention_sharded(q, k, v, Hs, out_full, rope=rope, op_type=op, stream=stream)
        else:
            ctx.self_attention(q, k, v, Hs, out_shard, rope=rope, op_type=op, stream=stream)

    def step_nccl():  # the unfused alternative: attention into the shard, then ncclAllGather + permute
        ctx.self_attention(q, k, v, Hs, out_shard, rope=rope, op_type=op, stream=stream)
        ctx.allgather_heads(out_shard.view(N, L, Hs, d), out_nccl.view(N, L, H, d), stream=stream)

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    if cfg.get("kind") in ("cross", "sparse"):
        if ws > 1:
            raise SystemExit("configs 2 and 4 are single-GPU measurements")
        line = run_other(args, cfg, ctx, kd_attn, torch, q, k, v, rope, op, out_dt, stream)
        print(json.dumps(line), flush=True)
        ctx.close()
        return

    if args.fa_only:
        qs = torch.empty(N, Hs, L, d, device=dev, dtype=torch.bfloat16 if op == kd_attn.BF16 else torch.float16)
        ks, vs = torch.empty_like(qs), torch.empty_like(qs)
        ctx.qk_prologue(q, k, v, qs, ks, vs, rope=rope, stream=stream)
        o4 = out_shard.view(N, L, Hs, d)
        for _ in range(max(args.warmup, 3)):
            ctx.flash_attn_ext(qs, ks, vs, o4, stream=stream)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            ctx.flash_attn_ext(qs, ks, vs, o4, stream=stream)
        b.record(stream)
        torch.cuda.synchronize()
        ctx.device_status()
        fms = a.elapsed_time(b) / args.steps
        if rank == 0:
            print(json.dumps({"fa_only": True, "workload": cfg["name"], "ms": fms,
                              "tflops": 4.0 * N * Hs * L * L * d / (fms * 1e-3) / 1e12}), flush=True)
        ctx.close()
        return

    for _ in range(max(args.warmup, 3)):
        step()
    ctx.device_status()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(node_gpus(local, ws) if local == 0 else []) as clk:
        # the sampler starts on local rank 0 only: align every rank after it is live, so no rank's
        # timed region contains another rank's sampler start-up
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    ctx.device_status()
    t = torch.tensor([ms], device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flop = 4.0 * N * H * L * L * d
    value = flop / (ms * 1e-3) / 1e12

    exchange = None
    if ws > 1:
        exchange = exchange_check(ctx, torch, dist, proj, out_full, rope, op, out_dt, ws, rank, N, L, Hs, Cs, dev,
                                  stream)

    nccl_ms = None
    if ws > 1:  # the same job with the exchange as a separate ncclAllGather + permute, for comparison
        out_nccl = torch.empty(N, L, H * d, device=dev, dtype=out_dt)
        for _ in range(2):
            step_nccl()
        barrier()
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0.record(stream)
        for _ in range(args.steps):
            step_nccl()
        n1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([n0.elapsed_time(n1) / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nccl_ms = float(t.item())
        del out_nccl

    # dominant kernel alone: flash attention on the bf16 operands the prologue produced
    qs = torch.empty(N, Hs, L, d, device=dev, dtype=torch.bfloat16 if op == kd_attn.BF16 else torch.float16)
    ks, vs = torch.empty_like(qs), torch.empty_like(qs)
    ctx.qk_prologue(q, k, v, qs, ks, vs, rope=rope, stream=stream)
    o4 = out_shard.view(N, L, Hs, d)
    for _ in range(2):
        ctx.flash_attn_ext(qs, ks, vs, o4, stream=stream)
    torch.cuda.synchronize()
    fa0, fa1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fa0.record(stream)
    for _ in range(args.steps):
        ctx.flash_attn_ext(qs, ks, vs, o4, stream=stream)
    fa1.record(stream)
    torch.cuda.synchronize()
    fa_ms = fa0.elapsed_time(fa1) / args.steps
    # prologue alone (HBM roofline): one launch for Q, K, V reading f32, writing 16-bit
    pr0, pr1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pr0.record(stream)
    for _ in range(args.steps):
        ctx.qk_prologue(q, k, v, qs, ks, vs, rope=rope, stream=stream)
    pr1.record(stream)
    torch.cuda.synchronize()
    pro_ms = pr0.elapsed_time(pr1) / args.steps
    del qs, ks, vs

    # end to end from pinned host buffers through the public API: kd_attn_self_attention_host
    # uploads, computes and downloads head group by head group, the copies of one group
    # overlapping the compute of the next.  With N > 1 ranks each rank carries its own heads'
    # columns from host memory to host memory (no device all-gather on this path).
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(out_shard.shape, dtype=out_dt).pin_memory()
    e2e_steps = max(1, min(args.e2e_steps, args.steps))

    def e2e_step():
        ctx.self_attention_host(hq, hk, hv, Hs, hout, rope=rope, op_type=op, stream=stream)

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    t = torch.tensor([e2e_ms], device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    h2d = 3 * N * L * Cs * 4
    d2h = hout.numel() * hout.element_size()
    if not torch.equal(hout[:, :64].to(dev), out_shard[:, :64]):
        raise SystemExit("host-buffer path disagrees with the device-buffer path")

    pk, pk_sus, pk_kind = peaks()
    fa_flop = 4.0 * N * Hs * L * L * d
    fa_tflops = fa_flop / (fa_ms * 1e-3) / 1e12
    traffic = profile_traffic()
    if traffic is not None and ws > 1:
        traffic = traffic / ws
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": cfg["op"],
        "data": "synthetic: seeded Philox4x32-10 N(0,1) projections generated on the device",
        "config": {"workload": cfg["name"], "global_batch": N, "seq_len": L, "heads": H, "head_dim": d,
                   "parallelism": f"heads{ws}" if ws > 1 else "single",
                   "step": ("kd_attn_self_attention_sharded (barrier, fused prologue, tcgen05 flash attention whose "
                            "epilogue stores every row into all ranks' symmetric copies over NVLink, barrier)")
                           if ws > 1 else
                           "kd_attn_self_attention (one fused RMSNorm+RoPE+cast prologue launch, tcgen05 flash attention)",
                   "l2": "inputs larger than L2 (3 x f32 projections per rank)"},
        "roofline": {"bound": "tensor", "achieved": fa_tflops, "peak": pk, "unit": "TFLOP/s",
                     "frac": fa_tflops / pk if pk else None, "peak_kind": f"{pk_kind} burst bf16",
                     "frac_of_sustained": fa_tflops / pk_sus if pk_sus else None,
                     "traffic": traffic, "kernel": "fmha_fwd_kernel<bf16>", "kernel_ms": fa_ms},
        "unfused_nccl_step_ms": nccl_ms,
        "prologue": {"ms": pro_ms, "gbs": (3 * N * L * Cs * 4 + 3 * N * L * Cs * 2) / (pro_ms * 1e-3) / 1e9},
        "e2e": {"value": flop / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "call": "kd_attn_self_attention_host (head-group pipelined H2D / compute / D2H)"},
        "gpu_launches": args.steps * 2,  # prologue + flash (the barriers are NCCL kernels)
        "clocks": clk.summary(),
    }
    if ws > 1:
        line["comm"] = {"backend": "nccl", "world_size": dist.get_world_size(), "gpus_active": ws,
                        "library_communicator_ranks": ws}
    if exchange is not None:
        line["exchange_check"] = exchange["status"]
        line["exchange_check_detail"] = exchange
    if ws == 1 and not args.no_extra:
        line["extra"] = extra_measurements(args, ctx, kd_attn, torch, q, k, v, rope, dev, stream)
    if rank == 0 and not args.no_cpu_baseline:
        cb = cpu_reference(cfg, seconds_target=args.ref_seconds)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if ws > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if exchange is not None and exchange["status"] != "pass":
        raise SystemExit("exchange_check failed: " + json.dumps(exchange))


if __name__ == "__main__":
    main()
