"""Benchmark: GQA decode tokens/s over the int4-compressed KV cache (B200).

Workload (Llama-3-8B decode layer): batch 64, 32 query /
8 KV heads, head_dim 128, context 8192 (8191 cached tokens + the new one),
bf16 activations, PolarQuant int4 KV cache, RoPE theta 500000.  One step is
one GroupQueryAttention operator call through the C ABI
(sa_group_query_attention): RoPE + quantize-on-append of the new token's K/V,
then attention of the 32 query heads over all 8192 cached tokens.  Inputs are
synthetic (seeded normal); the cache (604 MB) is larger than L2 (126 MB), so
no flush is needed between steps.

  value   tokens/s of the device-resident step (B / step time), max over ranks
  e2e     same metric through the same C-ABI call with q/k/v copied from
          pinned host memory and attn_out copied back inside the timed region
          (copy-in of the next step and copy-out of the previous one overlap the
          compute, as a serving loop runs them; the serial loop is reported beside it)
  roofline  the attention call alone (prep + decode + merge launches): algorithmic bytes / call time
  cpu_baseline  the CPU oracle (C restatement of the reference's Rust CPU
          path: encode + read_k/read_v + SDPA) on a bounded sample, rank 0

``--impl reference`` times that CPU restatement (all host threads) as the
reference arm.  ``--gpus N`` under torchrun: each rank decodes its own batch of
64 sequences (batch sharding, no collective; weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, HQ, HKV, D, T, BITS, THETA = 64, 32, 8, 128, 8192, 4, 500000.0
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one attention call on this
# workload, from one ncu capture of its three launches: prep 0.56 MB, decode_stream
# 606.68 + 5.75 MB, merge 5.97 MB (cold-cache reads of the partial records).
NCU_TRAFFIC_PER_CALL = 618_963_456
NCU_TRAFFIC_DECODE_STREAM = 612_429_312
CB = D * BITS // 8
METRIC = "GQA decode tokens/s over int4-compressed KV (Llama-3-8B layer, B=64, T=8192)"
UNIT = "tokens/s"
WORKLOAD = "llama3-8b-layer-decode (BASELINE config 3)"

# --config c5: the Llama-3-70B-shaped layer: 64 query / 8 KV
# heads (8 per KV head), batch 128, context 32768; 4.8 GB of int4 cache.
CONFIGS = {
    "c3": dict(B=64, HQ=32, HKV=8, D=128, T=8192, BITS=4, THETA=500000.0, METRIC=METRIC, WORKLOAD=WORKLOAD,
               NCU_TRAFFIC_PER_CALL=NCU_TRAFFIC_PER_CALL, NCU_TRAFFIC_DECODE_STREAM=NCU_TRAFFIC_DECODE_STREAM,
               KERNEL_NOTE="gqa attend call: decode_prep + decode_stream + decode_merge (decode_stream is 88% of "
                           "the call's device time)"),
    "c5": dict(B=128, HQ=64, HKV=8, D=128, T=32768, BITS=4, THETA=500000.0,
               METRIC="GQA decode tokens/s over int4-compressed KV (Llama-3-70B layer, B=128, T=32768)",
               WORKLOAD="llama3-70b-layer-decode (BASELINE config 5)", NCU_TRAFFIC_PER_CALL=None,
               NCU_TRAFFIC_DECODE_STREAM=None,
               KERNEL_NOTE="gqa attend call: decode_prep8 + decode8_stream + decode_merge<8>"),
}


def select_config(name):
    """Point the module's workload constants at BASELINE config `name`."""
    g = globals()
    g.update(CONFIGS[name])
    g["CB"] = g["D"] * g["BITS"] // 8


def algorithmic_bytes(b=None, hkv=None, t=None, hq=None, d=None, cb=None, act=2):
    """Per step: K+V codes and {scale, zp} of every cached token, q in, out, appended vectors."""
    b, hkv, t, hq, d, cb = (x if x is not None else y for x, y in zip((b, hkv, t, hq, d, cb),
                                                                     (B, HKV, T, HQ, D, CB)))
    cache = 2 * b * hkv * t * (cb + 8)
    return cache + b * hq * d * act * 2 + 2 * b * hkv * (cb + 8)


def attend_bytes(b=None, hkv=None, t=None, hq=None, d=None, cb=None, act=2):
    b, hkv, t, hq, d, cb = (x if x is not None else y for x, y in zip((b, hkv, t, hq, d, cb),
                                                                     (B, HKV, T, HQ, D, CB)))
    return 2 * b * hkv * t * (cb + 8) + b * hq * d * act * 2


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        self.gpu_id = gpu_id

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_uuid(torch, dev):
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index)


def build_workload(torch, sa, dev, seed, kv_begin=0, kv_count=None):
    """Cache filled with T-1 tokens (seeded), plus the step's q/k/v.

    ``kv_begin``/``kv_count`` select a shard of the KV heads (and their query
    heads) for the head-sharded mode.
    """
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    std = 1.28  # N(0,1) activations through N(0, 0.02) projections of width 4096
    kv_count = HKV if kv_count is None else kv_count
    hkv, hq = kv_count, kv_count * (HQ // HKV)
    cache = sa.GpuKvCache(1, HKV, D, T, batch=B, num_heads=HQ, bits=BITS, kv_head_begin=kv_begin,
                          kv_head_count=kv_count, device=dev)
    cos_np, sin_np = rope_np(T, D, THETA)
    cos = torch.from_numpy(cos_np).to(dev)
    sin = torch.from_numpy(sin_np).to(dev)
    chunk = 512
    pos = 0
    while pos < T - 1:
        n = min(chunk, T - 1 - pos)
        k = (torch.randn(B, n, hkv * D, device=dev, generator=g) * std).to(torch.bfloat16)
        v = (torch.randn(B, n, hkv * D, device=dev, generator=g) * std).to(torch.bfloat16)
        cache.append(0, k, v, cos_cache=cos, sin_cache=sin, do_rotary=True)
        cache.advance_position(n)
        pos += n
    q = (torch.randn(B, 1, hq * D, device=dev, generator=g) * std).to(torch.bfloat16)
    k = (torch.randn(B, 1, hkv * D, device=dev, generator=g) * std).to(torch.bfloat16)
    v = (torch.randn(B, 1, hkv * D, device=dev, generator=g) * std).to(torch.bfloat16)
    torch.cuda.synchronize(dev)
    return cache, cos, sin, q, k, v


def rope_np(rows, d, theta):
    half = d // 2
    inv = 1.0 / (theta ** (np.arange(half, dtype=np.float64) * 2.0 / d))
    ang = np.arange(rows, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def parity_sample(torch, cache, q, k, out, cos_np, sin_np, kv_count, rows):
    """Check the timed step's own output against the CPU oracle on a sample of batch rows.

    Runs after the timed region.  The cache then holds every token the last step attended to,
    the newest (appended by that step at position T-1) included.  Checks (1) the newest
    token's K codes and metadata bit for bit against PolarQuantizer::encode of RoPE(k), and
    (2) the attention output of every query head of the sampled rows against the composite
    oracle (read_k/read_v of all T tokens + causal SDPA) within 1e-3 + half a bf16 ulp.
    """
    import oracle  # the checker

    hq = kv_count * (HQ // HKV)
    rows = sorted(set(r for r in rows if 0 <= r < B))
    view = cache.view(0)
    kc = view.k_codes[rows, :, :T].cpu().numpy()
    km = view.k_meta[rows, :, :T].cpu().numpy()
    vc = view.v_codes_tokens()[rows][:, :, :T].cpu().numpy()
    vm = view.v_meta[rows, :, :T].cpu().numpy()
    signs = view.signs.cpu().numpy().astype(np.int8)
    nt = os.cpu_count() or 1
    # (1) the step's append: RoPE(k) at T-1, then PolarQuantizer::encode per KV head
    kn = k[rows].float().cpu().numpy().reshape(len(rows), 1, kv_count, D).transpose(0, 2, 1, 3)
    kr = oracle.apply_rope(np.ascontiguousarray(kn), cos_np, sin_np, np.array([T - 1]))
    codes_ok = True
    for h in range(kv_count):
        c, m = oracle.polar_encode_many(kr[:, h, 0], BITS, signs[h], nthreads=nt)
        codes_ok &= bool(np.array_equal(c, kc[:, h, T - 1]) and
                         np.array_equal(m.view(np.uint32), km[:, h, T - 1].view(np.uint32)))
    # (2) attention of the sampled rows
    qn = q[rows].float().cpu().numpy().reshape(len(rows), 1, hq, D).transpose(0, 2, 1, 3)
    qr = oracle.apply_rope(np.ascontiguousarray(qn), cos_np, sin_np, np.array([T - 1]))
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(D)))
    want = oracle.compressed_gqa(qr, kc, km, vc, vm, signs, BITS, scale, nthreads=nt)
    got = out[rows].float().cpu().numpy().reshape(want.shape)
    err = np.abs(got - want)
    bound = 1e-3 + np.abs(want) * 2.0 ** -8
    return {"max_abs": float(err.max()), "ok": bool(np.all(err <= bound)) and codes_ok,
            "codes_bit_exact": codes_ok, "rows": rows, "units": len(rows) * kv_count,
            "bar": "max-abs 1e-3 + half a bf16 ulp vs the composite CPU oracle; newest token's codes bit-exact"}


def cpu_oracle_step_time(cache_view_np, q_np, k_new, v_new, signs, units, nthreads):
    """One CPU step of the reference path on `units` (b, kv_head) pairs:
    encode the new token (write_kv) + read_k/read_v of all T tokens + SDPA."""
    import oracle

    kc, km, vc, vm = cache_view_np
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(D)))
    t0 = time.perf_counter()
    # append: PolarQuantizer::encode of the new K and V of every sampled unit
    for u in range(units):
        b, h = divmod(u, HKV)
        oracle.polar_encode(k_new[b, h], BITS, signs[h])
        oracle.polar_encode(v_new[b, h], BITS, signs[h])
    nb = (units + HKV - 1) // HKV
    oracle.compressed_gqa(q_np[:nb], kc[:nb], km[:nb], vc[:nb], vm[:nb], signs, BITS, scale, nthreads=nthreads,
                          unit_begin=0, unit_end=units)
    return time.perf_counter() - t0


def cpu_sample(torch, cache, q, k, v, dev, target_s=10.0, nthreads=1):
    """Bounded CPU sample of the same workload; returns (tokens/s, sample description)."""
    view = cache.view(0)
    nb = 2  # batch rows copied to host (16 units)
    kc = view.k_codes[:nb, :, :T].cpu().numpy()
    km = view.k_meta[:nb, :, :T].cpu().numpy()
    vc = view.v_codes_tokens()[:nb, :, :T].cpu().numpy()
    vm = view.v_meta[:nb, :, :T].cpu().numpy()
    signs = view.signs.cpu().numpy().astype(np.int8)
    qn = q.float().cpu().numpy().reshape(B, 1, HQ, D).transpose(0, 2, 1, 3)[:nb].copy()
    kn = k.float().cpu().numpy().reshape(B, HKV, D)
    vn = v.float().cpu().numpy().reshape(B, HKV, D)
    data = (kc, km, vc, vm)
    per_unit = cpu_oracle_step_time(data, qn, kn, vn, signs, 1, 1)
    units = int(max(1, min(nb * HKV, target_s * nthreads / max(per_unit, 1e-6))))
    if nthreads > 1:
        units = max(units, min(nb * HKV, nthreads))
    dt = cpu_oracle_step_time(data, qn, kn, vn, signs, units, nthreads)
    total_units = B * HKV
    step_time = dt * total_units / units
    desc = (f"{units} of {total_units} (batch row, kv head) units of the full step (T={T}), {nthreads} thread(s), "
            f"scaled by {total_units}/{units}; C restatement of the reference Rust CPU path (-O2, no FMA)")
    return B / step_time, desc


def reference_step(data, q_new, k_new, v_new, signs, cos_np, sin_np, units, nthreads):
    """One step of the reference CPU path on the first ``units`` (row, KV head) units, timed:
    RoPE of q and k at position T-1 (apply_rope_in_place), PolarQuantizer::encode of the new
    K and V into the cache (write_kv), then read_k/read_v of all T tokens and causal SDPA
    (the composite oracle), all host threads."""
    import oracle

    kc, km, vc, vm = data
    nb = (units + HKV - 1) // HKV
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(D)))
    t0 = time.perf_counter()
    pos = np.array([T - 1])
    qr = oracle.apply_rope(q_new[:nb], cos_np, sin_np, pos)   # (nb, HQ, 1, D)
    kr = oracle.apply_rope(k_new[:nb], cos_np, sin_np, pos)   # (nb, HKV, 1, D)
    for h in range(HKV):
        c, m = oracle.polar_encode_many(kr[:, h, 0], BITS, signs[h], nthreads=nthreads)
        kc[:nb, h, T - 1], km[:nb, h, T - 1] = c, m
        c, m = oracle.polar_encode_many(v_new[:nb, h, 0], BITS, signs[h], nthreads=nthreads)
        vc[:nb, h, T - 1], vm[:nb, h, T - 1] = c, m
    out = oracle.compressed_gqa(qr, kc[:nb], km[:nb], vc[:nb], vm[:nb], signs, BITS, scale, nthreads=nthreads,
                                unit_begin=0, unit_end=units)
    return time.perf_counter() - t0, out


def reference_inputs():
    """The GPU arm's step inputs, staged to host memory before any timing: the cache after
    its T-1 seeded appends (rank 0's seed) and the step's q/k/v.  On a machine without a GPU
    the same shapes are generated on the host and encoded with the CPU restatement."""
    import oracle

    try:
        import torch

        have_gpu = torch.cuda.is_available()
    except ImportError:
        have_gpu = False
    if have_gpu:
        import smallaios_b200 as sa

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        cache, _, _, q, k, v = build_workload(torch, sa, dev, seed=1000)
        view = cache.view(0)
        data = (view.k_codes[:, :, :T].cpu().numpy(), view.k_meta[:, :, :T].cpu().numpy(),
                view.v_codes_tokens()[:, :, :T].cpu().numpy(), view.v_meta[:, :, :T].cpu().numpy())
        signs = view.signs.cpu().numpy().astype(np.int8)
        qn = q.float().cpu().numpy().reshape(B, 1, HQ, D).transpose(0, 2, 1, 3).copy()
        kn = k.float().cpu().numpy().reshape(B, 1, HKV, D).transpose(0, 2, 1, 3).copy()
        vn = v.float().cpu().numpy().reshape(B, 1, HKV, D).transpose(0, 2, 1, 3).copy()
        cache.close()
        src = "the GPU arm's own cache bytes (rank 0's seed, T-1 tokens appended), copied to host"
    else:
        rng = np.random.default_rng(1000)
        signs = oracle.cache_signs(oracle.DEFAULT_SEED, 1, HKV, D)[0]
        cos_np, sin_np = rope_np(T, D, THETA)
        kc = np.zeros((B, HKV, T, CB), np.uint8)
        vc = np.zeros_like(kc)
        km = np.zeros((B, HKV, T, 2), np.float32)
        vm = np.zeros_like(km)
        for b in range(B):
            kx = (rng.standard_normal((1, HKV, T - 1, D)) * 1.28).astype(np.float32)
            vx = (rng.standard_normal((HKV, T - 1, D)) * 1.28).astype(np.float32)
            kx = oracle.apply_rope(kx, cos_np, sin_np, np.arange(T - 1))[0]
            for h in range(HKV):
                kc[b, h, :T - 1], km[b, h, :T - 1] = oracle.polar_encode_many(kx[h], BITS, signs[h])
                vc[b, h, :T - 1], vm[b, h, :T - 1] = oracle.polar_encode_many(vx[h], BITS, signs[h])
        data = (kc, km, vc, vm)
        qn = (rng.standard_normal((B, HQ, 1, D)) * 1.28).astype(np.float32)
        kn = (rng.standard_normal((B, HKV, 1, D)) * 1.28).astype(np.float32)
        vn = (rng.standard_normal((B, HKV, 1, D)) * 1.28).astype(np.float32)
        src = "seeded host normals (std 1.28) encoded by the CPU restatement (no GPU on this machine)"
    return data, qn, kn, vn, signs, src


def run_reference(args):
    """--impl reference: the CPU restatement of the reference path, all host threads, rank 0 only.

    Every timed step is the whole reference step over all B x Hkv units (RoPE, write_kv of the
    new token, read_k/read_v of T tokens, SDPA) unless that would not fit a few minutes; then
    each step runs a fixed subset of units and the line says so.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle

    oracle.build()
    nthreads = os.cpu_count() or 1
    data, qn, kn, vn, signs, src = reference_inputs()
    cos_np, sin_np = rope_np(T, D, THETA)
    total = B * HKV
    # one probe step on a thread's worth of units sizes the run
    probe_units = min(total, max(HKV, nthreads))
    dt, _ = reference_step(data, qn, kn, vn, signs, cos_np, sin_np, probe_units, nthreads)
    est_full = dt * total / probe_units
    budget_s = 240.0
    units = total
    if est_full * (args.steps + args.warmup) > budget_s:
        units = max(probe_units, int(budget_s / (args.steps + args.warmup) / dt * probe_units) // HKV * HKV)
        units = min(units, total)
    for _ in range(args.warmup):
        reference_step(data, qn, kn, vn, signs, cos_np, sin_np, units, nthreads)
    times = [reference_step(data, qn, kn, vn, signs, cos_np, sin_np, units, nthreads)[0] for _ in range(args.steps)]
    measured = float(np.mean(times))
    step = measured * total / units
    value = B / step
    if units == total:
        sample = (f"every step is the full step: all {total} (batch row, kv head) units, T={T}, on {src}; "
                  f"the C restatement of the reference Rust CPU path (-O2, no FMA; no rustc here), "
                  f"{nthreads} threads")
    else:
        sample = (f"{units} of {total} (batch row, kv head) units per step (a full step would not fit the run), "
                  f"scaled by {total}/{units}; T={T}, on {src}; the C restatement of the reference Rust CPU path, "
                  f"{nthreads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded normal, std 1.28)",
        "config": {"workload": WORKLOAD, "batch_per_gpu": B, "global_batch": B, "q_heads": HQ, "kv_heads": HKV,
                   "head_dim": D, "context": T, "kv_bits": BITS, "rope_theta": THETA},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads,
                         "kind": "port" if units == total else "port (sampled, scaled)", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "measured_s_per_step": measured, "units_per_step": units,
    }
    print(json.dumps(line), flush=True)
    return 0


# MatMulNBits: K=4096, N=14336, block 32, fp16 scales, zero point 8.
MNB_K, MNB_N, MNB_BLOCK = 4096, 14336, 32


def mnb_bytes(m, n=MNB_N, k=MNB_K, block=MNB_BLOCK):
    """Codes + fp16 scales + fp16 A in + fp16 Y out."""
    return n * k // 2 + n * (k // block) * 2 + m * k * 2 + m * n * 2


def run_matmul_nbits(args):
    """``--workload matmul_nbits``: one MatMulNBits call on config 2 per step (not the headline).

    Six weight sets are cycled so that every call streams its 33 MB of codes
    and scales from HBM (six sets, 198 MB, exceed the 126 MB L2).
    """
    import torch

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    m, n, k, blk = args.m, MNB_N, MNB_K, MNB_BLOCK
    sets = []
    for _ in range(6):
        codes = torch.randint(0, 256, (n, k // blk, blk // 2), dtype=torch.uint8, device=dev, generator=g)
        scales = (torch.rand(n, k // blk, device=dev, generator=g) * 0.015 + 0.005).half()
        sets.append((codes, scales))
    a = torch.randn(m, k, device=dev, generator=g).half()
    y = torch.empty(m, n, dtype=torch.half, device=dev)
    stream = torch.cuda.current_stream(dev)
    packed = [sa.PackedNBitsWeight(c, s, K=k, N=n, block_size=blk) for c, s in sets] if args.packed else None

    def call(i):
        if packed is not None:
            sa.matmul_nbits_packed(a, packed[i % 6], out=y)
        else:
            c, s = sets[i % 6]
            sa.matmul_nbits(a, c, s, K=k, N=n, block_size=blk, out=y)

    for i in range(max(args.warmup, 3)):
        call(i)
    torch.cuda.synchronize(dev)
    # six calls (one per weight set) captured as a CUDA graph and replayed: the
    # device time of back-to-back calls, without the host's per-call cost
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(6):
                call(i)
        graph.replay()
        torch.cuda.synchronize(dev)
    reps = max(1, args.steps // 6) if graph is not None else args.steps
    l0 = lib.sa_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        if graph is not None:
            graph.replay()
        else:
            call(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    calls = reps * 6 if graph is not None else reps
    launches = lib.sa_kernel_launches() - l0 if graph is None else calls
    t_ms = e0.elapsed_time(e1) / calls
    peak, peak_kind = load_peaks()
    byts = mnb_bytes(m)
    flops = 2.0 * m * n * k
    achieved = byts / (t_ms * 1e-3) / 1e9
    line = {"metric": f"MatMulNBits int4 GEMV/GEMM time (K={k}, N={n}, M={m}, block {blk}, fp16)",
            "value": t_ms * 1e3, "unit": "us", "higher_is_better": False, "n_gpus": 1, "steps": calls,
            "warmup": max(args.warmup, 3), "ms_per_step": t_ms, "dtype": "int4-w/fp16-act/f32-acc",
            "data": "synthetic (codes U{0..255} bytes, scales U[0.005, 0.02])",
            "config": {"workload": "matmul-nbits (BASELINE config 2)", "m": m, "n": n, "k": k, "block": blk,
                       "weights": "prepacked (sa_matmul_nbits_prepack)" if args.packed else "ORT layout",
                       "launch": "host launches" if graph is None else "CUDA graph of six calls, replayed",
                       "l2": "six weight sets cycled (198 MB > L2)"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "algorithmic_bytes": byts, "tflops": flops / (t_ms * 1e-3) / 1e12,
                         "peak_source": f"{peak_kind} hbm_gbs"}}
    print(json.dumps(line), flush=True)


def run_decode_block(args):
    """``--workload decode_block``: the attention block of one decode layer (not the headline).

    One step = the fused QKV projection (sa_qkv_project_append: int4
    MatMulNBits of the packed Wq/Wk/Wv, RoPE, quantize-on-append) + the
    attention over the cache (sa_gqa_attend on the rotated q).  The line also
    times the unfused sequence on the same inputs: MatMulNBits of the packed
    weights, then GroupQueryAttention (RoPE + append + attention).
    Weights are random int4 codes with scales U[0.005, 0.02] (hidden 4096,
    block 32), activations N(0, 1); the cache is the headline's.
    """
    import torch

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cache, cos, sin, _, _, _ = build_workload(torch, sa, dev, seed=1)
    hidden = 4096 if args.config == "c3" else 8192
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    n = (HQ + 2 * HKV) * D
    codes = torch.randint(0, 256, (n, hidden // 32, 16), dtype=torch.uint8, device=dev, generator=g)
    scales = (torch.rand(n, hidden // 32, device=dev, generator=g) * 0.015 + 0.005).to(torch.bfloat16)
    x = torch.randn(B, hidden, device=dev, generator=g).to(torch.bfloat16)
    q = torch.empty(B, HQ * D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, HKV * D, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    y = torch.empty(B, n, dtype=torch.bfloat16, device=dev)
    out = torch.empty(B, 1, HQ * D, dtype=torch.bfloat16, device=dev)

    def fused():
        cache.set_position(T - 1)
        sa.qkv_project_append(x, codes, scales, cache, 0, cos_cache=cos, sin_cache=sin, q_out=q, k_out=k, v_out=v)
        sa.gqa_attend(q.view(B, 1, HQ * D), cache, 0, num_heads=HQ, do_rotary=False, out=out)

    def unfused():
        cache.set_position(T - 1)
        sa.matmul_nbits(x, codes, scales, K=hidden, N=n, out=y)
        q.copy_(y[:, :HQ * D])
        k.copy_(y[:, HQ * D:(HQ + HKV) * D])
        v.copy_(y[:, (HQ + HKV) * D:])
        sa.group_query_attention(q.view(B, 1, -1), k.view(B, 1, -1), v.view(B, 1, -1), cache, 0, num_heads=HQ,
                                 kv_num_heads=HKV, cos_cache=cos, sin_cache=sin, out=out)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        c0 = lib.sa_kernel_launches()
        with torch.cuda.graph(graph):
            fn()
        launches = lib.sa_kernel_launches() - c0
        for _ in range(args.warmup):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / args.steps, launches

    sampler = ClockSampler(gpu_uuid(torch, dev))
    sampler.start()
    t_ms, launches = timed(fused)
    clocks = sampler.stop()
    u_ms, u_launches = timed(unfused)
    peak, peak_kind = load_peaks()
    wbytes = n * hidden // 2 + n * (hidden // 32) * 2
    byts = wbytes + B * hidden * 2 + attend_bytes() + 2 * B * HKV * (CB + 8)
    line = {
        "metric": f"attention block tokens/s (fused QKV MatMulNBits + RoPE + append + attention), {WORKLOAD}",
        "value": B / (t_ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4-w/int4-kv/bf16-act/f32-acc", "data": "synthetic (seeded; random int4 weights)",
        "config": {"workload": f"decode attention block, {WORKLOAD}", "batch": B, "hidden": hidden, "q_heads": HQ,
                   "kv_heads": HKV, "head_dim": D, "context": T, "launch": "CUDA graph of one step, replayed"},
        "gpu_launches": int(launches) * args.steps,
        "unfused": {"ms_per_step": u_ms, "value": B / (u_ms * 1e-3), "launches_per_step": int(u_launches),
                    "sequence": "sa_matmul_nbits (QKV) + sa_group_query_attention"},
        "roofline": {"bound": "hbm", "achieved": byts / (t_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": byts / (t_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": byts, "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs"},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    cache.close()
    return 0


def run_decode_layer(args):
    """``--workload decode_layer``: one whole decoder layer per step (not the headline).

    smallaios_b200.decoder_layer_step: SkipSimplifiedLayerNormalization, the
    fused QKV projection (RoPE + append), attention over the cache, o_proj,
    SkipSimplifiedLayerNormalization, the packed gate|up projection, SwiGLU,
    down_proj; all projections int4 MatMulNBits (random codes, scales
    U[0.005, 0.02], block 32), the cache is the headline's.
    """
    import torch

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cache, cos, sin, _, _, _ = build_workload(torch, sa, dev, seed=1)
    hidden, inter = (4096, 14336) if args.config == "c3" else (8192, 28672)
    g = torch.Generator(device=dev)
    g.manual_seed(5)

    def weight(n, k):
        codes = torch.randint(0, 256, (n, k // 32, 16), dtype=torch.uint8, device=dev, generator=g)
        scales = (torch.rand(n, k // 32, device=dev, generator=g) * 0.015 + 0.005).to(torch.bfloat16)
        return codes, scales

    qkv = weight((HQ + 2 * HKV) * D, hidden)
    wo = weight(hidden, HQ * D)
    wgu = weight(2 * inter, hidden)
    wdn = weight(hidden, inter)
    ones = torch.ones(hidden, dtype=torch.bfloat16, device=dev)
    w = sa.LayerWeights(*qkv, *wo, *wgu, *wdn, ones, ones, 1e-5)
    x = torch.randn(B, hidden, device=dev, generator=g).to(torch.bfloat16)
    resid = torch.randn(B, hidden, device=dev, generator=g).to(torch.bfloat16)

    def step():
        cache.set_position(T - 1)
        sa.decoder_layer_step(x, resid, w, cache, 0, cos_cache=cos, sin_cache=sin)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    c0 = lib.sa_kernel_launches()
    with torch.cuda.graph(graph):
        step()
    launches = lib.sa_kernel_launches() - c0
    for _ in range(args.warmup):
        graph.replay()
    sampler = ClockSampler(gpu_uuid(torch, dev))
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    t_ms = e0.elapsed_time(e1) / args.steps
    peak, peak_kind = load_peaks()
    wbytes = sum(c.numel() + s.numel() * 2 for c, s in (qkv, wo, wgu, wdn))
    byts = wbytes + attend_bytes() + 2 * B * HKV * (CB + 8) + 12 * B * hidden * 2
    line = {
        "metric": f"decoder layer tokens/s (one full decode-step layer), {WORKLOAD}",
        "value": B / (t_ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4-w/int4-kv/bf16-act/f32-acc", "data": "synthetic (seeded; random int4 weights)",
        "config": {"workload": f"decoder layer, {WORKLOAD}", "batch": B, "hidden": hidden, "intermediate": inter,
                   "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context": T,
                   "launch": "CUDA graph of one step, replayed"},
        "gpu_launches": int(launches) * args.steps, "launches_per_step": int(launches),
        "roofline": {"bound": "hbm", "achieved": byts / (t_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": byts / (t_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": byts, "weight_bytes": wbytes,
                     "traffic": None, "peak_source": f"{peak_kind} hbm_gbs"},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    graph.reset()
    cache.close()
    return 0


def run_prefill_stack(args):
    """``--workload prefill_stack``: BASELINE config 4, the whole 32-layer prefill forward.

    B = 8 prompts of 2048 tokens (token ids uniform in a 128256 vocabulary, an embedding
    table of random bf16 rows), 32 Llama-3-8B layers (hidden 4096, 32 query / 8 KV heads of
    128, intermediate 14336), each with its own random int4 MatMulNBits weights (block 32,
    codes U{0..255} bytes, scales U[0.005, 0.02]) and its own int8 layer of the KV cache.
    One step = the embedding gather, then prefill_layer_step for the 32 layers (RMSNorm, the
    Q/K/V, o, gate|up and down MatMulNBits of 16384 rows on tcgen05, RoPE + quantize-on-append
    of the prompts, the causal prefill attention, SwiGLU); no LM head.  Roofline: tensor, the
    algorithmic FLOPs of the projections (2*M*N*K each) and of the causal attention
    (4*B*Hq*S*S/2*D) against the measured bf16 peak.
    """
    import torch

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    b, s, hq, hkv, d, bits = 8, 2048, 32, 8, 128, 8
    hidden, inter, layers, vocab = 4096, 14336, args.layers, 128256
    m = b * s
    cos_np, sin_np = rope_np(s + 8, d, THETA)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    cache = sa.GpuKvCache(layers, hkv, d, s + 8, batch=b, num_heads=hq, bits=bits, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(11)

    def weight(n, k):
        codes = torch.randint(0, 256, (n, k // 32, 16), dtype=torch.uint8, device=dev, generator=g)
        scales = (torch.rand(n, k // 32, device=dev, generator=g) * 0.015 + 0.005).to(torch.bfloat16)
        return codes, scales

    ones = torch.ones(hidden, dtype=torch.bfloat16, device=dev)
    ws = [sa.LayerWeights(*weight((hq + 2 * hkv) * d, hidden), *weight(hidden, hq * d), *weight(2 * inter, hidden),
                          *weight(hidden, inter), ones, ones, 1e-5) for _ in range(layers)]
    table = (torch.randn(vocab, hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    tokens = torch.randint(0, vocab, (m,), device=dev, generator=g)

    def step():
        x = torch.index_select(table, 0, tokens)
        resid = None
        for li in range(layers):
            cache.set_position(0)
            x, resid = sa.prefill_layer_step(x, resid, ws[li], cache, li, batch=b, seq_len=s, cos_cache=cos,
                                             sin_cache=sin)
        return x

    warm = max(args.warmup, 3)
    for _ in range(warm):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_uuid(torch, dev))
    sampler.start()
    l0 = lib.sa_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    launches = lib.sa_kernel_launches() - l0
    t_ms = e0.elapsed_time(e1) / args.steps
    finite = bool(torch.isfinite(out).all().item())
    proj = 2.0 * m * hidden * ((hq + 2 * hkv) * d + 2 * inter) + 2.0 * m * hq * d * hidden + 2.0 * m * inter * hidden
    attn = 4.0 * b * hq * s * s / 2 * d
    flops = layers * (proj + attn)
    peak_tf, peak_kind = 1590.0, "fallback 1590 TFLOP/s"
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            v = float(json.load(f).get("bf16_tflops_sustained", 0) or 0)
        if v:
            peak_tf, peak_kind = v, "measured bf16_tflops_sustained (a seconds-long step)"
    achieved = flops / (t_ms * 1e-3) / 1e12
    line = {
        "metric": "prefill tokens/s, 32-layer Llama-3-8B stack (BASELINE config 4)",
        "value": m / (t_ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": warm,
        "ms_per_step": t_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4-w/int8-kv/bf16-act/f32-acc",
        "data": "synthetic (random token ids, random embedding rows and int4 weights)",
        "config": {"workload": "llama3-8b 32-layer prefill (BASELINE config 4)", "batch": b, "prompt": s,
                   "layers": layers, "hidden": hidden, "intermediate": inter, "q_heads": hq, "kv_heads": hkv,
                   "head_dim": d, "kv_bits": bits, "lm_head": False, "launch": "host launches",
                   "l2": "activations of 16384 rows and 123 MB of weights per layer exceed L2"},
        "gpu_launches": int(launches),
        "output_finite": finite,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "algorithmic_flops": flops, "projection_flops": layers * proj,
                     "attention_flops": layers * attn, "traffic": None, "peak_source": peak_kind},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    cache.close()
    return 0


def run_prefill_attention(args):
    """``--workload prefill``: the attention of the C4 prefill (not the headline).

    One step = one GroupQueryAttention call on a whole prompt per sequence
    (B = 8, S = 2048, 32 query / 8 KV heads, D = 128, int8 KV, theta 5e5):
    quantize-on-append of the 2048 tokens, then causal attention of the 2048
    queries on the tcgen05 prefill kernel.  Roofline: tensor (causal
    attention FLOPs 4*B*Hq*S*S/2*D against the measured bf16 peak; the kernel
    computes in fp16 with f32 accumulation, twice over for the hi + lo halves).
    """
    import torch

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    b, s, hq, hkv, d, bits = 8, 2048, 32, 8, 128, 8
    cos_np, sin_np = rope_np(s + 8, d, THETA)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    cache = sa.GpuKvCache(1, hkv, d, s + 8, batch=b, num_heads=hq, bits=bits, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    q = (torch.randn(b, s, hq * d, device=dev, generator=g) * 1.28).to(torch.bfloat16)
    k = (torch.randn(b, s, hkv * d, device=dev, generator=g) * 1.28).to(torch.bfloat16)
    v = (torch.randn(b, s, hkv * d, device=dev, generator=g) * 1.28).to(torch.bfloat16)
    out = torch.empty_like(q)

    def step():
        cache.set_position(0)
        sa.group_query_attention(q, k, v, cache, 0, num_heads=hq, kv_num_heads=hkv, cos_cache=cos, sin_cache=sin,
                                 out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_uuid(torch, dev))
    sampler.start()
    l0 = lib.sa_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    launches = lib.sa_kernel_launches() - l0
    t_ms = e0.elapsed_time(e1) / args.steps
    flops = 4.0 * b * hq * s * s / 2 * d
    peak_tf = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak_tf = float(json.load(f).get("bf16_tflops", 0)) or None
    peak_kind = "measured bf16_tflops" if peak_tf else "fallback 1590 TFLOP/s"
    peak_tf = peak_tf or 1590.0
    achieved = flops / (t_ms * 1e-3) / 1e12
    line = {
        "metric": "prefill attention tokens/s (quantize-on-append + causal GQA of whole prompts), BASELINE config 4 shape",
        "value": b * s / (t_ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8-kv/bf16-act/fp16-tcgen05/f32-acc", "data": "synthetic (seeded normal, std 1.28)",
        "config": {"workload": "llama3-8b prefill attention, one layer (BASELINE config 4 shape)", "batch": b,
                   "prompt": s, "q_heads": hq, "kv_heads": hkv, "head_dim": d, "kv_bits": bits,
                   "launch": "host launches"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "algorithmic_flops": flops, "traffic": None,
                     "peak_source": peak_kind},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    cache.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the check of the timed step's output against the CPU oracle (after timing)")
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS),
                    help="gqa_decode shape: c3 = Llama-3-8B layer (the headline), c5 = Llama-3-70B layer")
    ap.add_argument("--batch", type=int, default=None,
                    help="gqa_decode: override the config's batch (a smaller case for profiler captures)")
    ap.add_argument("--workload", default="gqa_decode",
                    choices=["gqa_decode", "matmul_nbits", "decode_block", "decode_layer", "prefill", "prefill_stack"],
                    help="gqa_decode = the headline (config 3); matmul_nbits = config 2; decode_block = fused QKV projection + attention of one layer (with the unfused sequence timed beside it); decode_layer = a whole decoder layer; prefill = the C4 prefill attention; prefill_stack = the C4 32-layer prefill forward; one line, 1 GPU")
    ap.add_argument("--m", type=int, default=1, help="matmul_nbits rows (1 = decode GEMV, 64 = batched)")
    ap.add_argument("--layers", type=int, default=32, help="prefill_stack: decoder layers (config 4: 32)")
    ap.add_argument("--packed", action="store_true", help="matmul_nbits: weights prepacked once (m <= 8)")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every step from the host instead of replaying a CUDA graph of one step")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="heads mode: peer = the decode epilogue stores every rank's copy over NVLink "
                         "(symmetric memory) + one barrier; nccl = NCCL all-gather of attn_out")
    ap.add_argument("--no-heads", action="store_true",
                    help="N>1: time only the batch-sharded mode (by default the head-sharded mode is timed too)")
    ap.add_argument("--mode", default="batch", choices=["batch", "heads"],
                    help="N>1: batch = every rank decodes its own 64 sequences (weak scaling, no collective); "
                         "heads = the 64 sequences' KV heads split over the ranks, attn_out all-gathered over "
                         "NCCL (strong scaling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    select_config(args.config)
    if args.batch is not None:
        globals()["B"] = args.batch
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "matmul_nbits":
        return run_matmul_nbits(args)
    if args.workload == "decode_block":
        return run_decode_block(args)
    if args.workload == "decode_layer":
        return run_decode_layer(args)
    if args.workload == "prefill":
        return run_prefill_attention(args)
    if args.workload == "prefill_stack":
        return run_prefill_stack(args)

    return run_gqa_decode(args)


def measure_decode(args, torch, dist, sa, lib, dev, world, rank, local, *, heads, gather, e2e, cpu):
    """Build the workload, time it and check it; returns the measurements (max over ranks).

    heads=False: every rank decodes its own B sequences (batch sharding, no collective).
    heads=True (world > 1): the B sequences' KV heads are split over the ranks and attn_out is
    gathered ("peer": the decode merge stores every rank's copy over NVLink and completes the
    gather on the device; "nccl": NCCL all-gather after the local operator).
    """
    peer = None
    shard = None
    if heads:
        from smallaios_b200 import sharding

        shard = sharding.head_shard(HQ, HKV, world, rank)
        kv_count = shard.kv_count
        cache, cos, sin, q, k, v = build_workload(torch, sa, dev, seed=1000 + rank, kv_begin=shard.kv_begin,
                                                  kv_count=kv_count)
        gathered = torch.empty(B, 1, HQ * D, dtype=q.dtype, device=dev)
        peer = sharding.PeerGather((B, 1, HQ * D), q.dtype, dev) if gather == "peer" else None
    else:
        kv_count = HKV
        cache, cos, sin, q, k, v = build_workload(torch, sa, dev, seed=1000 + rank)
        gathered = None
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    last = {}

    def gqa(q_, k_, v_, out_=None, res_=None):
        """One operator call; returns the tensor holding the step's attn_out.  With the fused
        gather that is the gather buffer itself (valid until two steps later) unless `res_` asks
        for a copy, which the end-to-end loop makes before its copy-out stream reads it."""
        cache.set_position(T - 1)
        if heads:
            dst = gathered if res_ is None else res_
            res = sharding.sharded_group_query_attention(q_, k_, v_, cache, 0, num_heads=HQ, kv_num_heads=HKV,
                                                         shard=shard, cos_cache=cos, sin_cache=sin, do_rotary=True,
                                                         local_out=out, out=None if peer else dst, gather=peer)
            if peer is not None and res_ is not None:
                res_.copy_(res)
                res = res_
        else:
            res = out if out_ is None else out_
            sa.group_query_attention(q_, k_, v_, cache, 0, num_heads=HQ, kv_num_heads=HKV, cos_cache=cos,
                                     sin_cache=sin, do_rotary=True, out=res)
        last["res"] = res
        return res

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # Steps per CUDA graph: consecutive steps are captured together (as a serving loop captures a
    # forward pass), so successive steps' launches overlap through programmatic dependencies
    # instead of paying a graph launch each.  The fused gather alternates two buffer sets, so
    # there a graph holds an even number of steps.  The timed step count stays exactly --steps.
    spg = next(n for n in (10, 8, 6, 5, 4, 3, 2, 1)
               if args.steps % n == 0 and (peer is None or n % 2 == 0 or n == 1))
    if args.no_graph:
        spg = 1
    if peer is not None and spg % 2:
        spg = 2  # odd step counts round up to whole buffer pairs
    replays = (args.steps + spg - 1) // spg
    steps = replays * spg

    def step():
        for _ in range(spg):
            gqa(q, k, v)

    for _ in range(args.warmup):
        step()
    barrier()
    run, graph_launches, graph = step, None, None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        c0 = lib.sa_kernel_launches()
        with torch.cuda.graph(graph):
            step()
        graph_launches = lib.sa_kernel_launches() - c0
        run = graph.replay
        for _ in range(args.warmup):
            run()
        barrier()

    sampler = ClockSampler(gpu_uuid(torch, dev))
    sampler.start()
    launches0 = lib.sa_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(replays):
        run()
    e1.record(stream)
    barrier()
    launches = lib.sa_kernel_launches() - launches0 if graph_launches is None else graph_launches * replays
    t_ms = e0.elapsed_time(e1) / steps
    clocks = sampler.stop()

    # The attention call alone (prep + decode + merge, no append, no gather), for the roofline.
    for _ in range(3):
        cache.set_position(T - 1)
        sa.gqa_attend(q, cache, 0, num_heads=HQ, cos_cache=cos, sin_cache=sin, do_rotary=True, out=out)
    torch.cuda.synchronize(dev)
    la0 = lib.sa_kernel_launches()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.steps):
        sa.gqa_attend(q, cache, 0, num_heads=HQ, cos_cache=cos, sin_cache=sin, do_rotary=True, out=out)
    a1.record(stream)
    torch.cuda.synchronize(dev)
    attend_launches = (lib.sa_kernel_launches() - la0) // args.steps
    attend_ms = a0.elapsed_time(a1) / args.steps

    e2e_res = None
    if e2e:
        e2e_res = measure_e2e(args, torch, sa, dev, stream, barrier, cache, cos, sin, q, k, v, out, gqa, heads,
                              gathered, spg)
    if heads:  # the last timed step's output again (the roofline loop above wrote only `out`)
        step()
        torch.cuda.synchronize(dev)

    parity = None
    if not args.no_parity:
        torch.cuda.synchronize(dev)
        res = out
        if heads:  # the rank's own heads of the gathered output of the last step
            res = last["res"][..., shard.q_begin * D:(shard.q_begin + shard.q_count) * D]
        cos_np, sin_np = rope_np(T, D, THETA)
        parity = parity_sample(torch, cache, q, k, res, cos_np, sin_np, kv_count, [0, B // 2, B - 1])

    status = cache.device_status(clear=True)

    # max over ranks (every rank takes the same collective steps)
    e2e_ms = e2e_res["graph_ms_per_step"] if e2e_res else -1.0
    e2e_host_ms = e2e_res["host_ms_per_step"] if e2e_res else -1.0
    e2e_serial_ms = e2e_res["serial_ms_per_step"] if e2e_res else -1.0
    pmax = -1.0 if parity is None else parity["max_abs"]
    pbad = 0.0 if parity is None or parity["ok"] else 1.0
    vals = torch.tensor([t_ms, e2e_ms, attend_ms, e2e_host_ms, e2e_serial_ms, pmax, pbad, float(status)],
                        device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, attend_ms, e2e_host_ms, e2e_serial_ms, pmax, pbad, status = vals.tolist()
    if parity is not None:
        parity.update(max_abs=pmax, ok=pbad == 0.0, ranks=world)
    if e2e_res:
        # both pipelines copy every step's data in and out; the faster (each the max over ranks) is
        # the reported e2e
        e2e_res.update(ms_per_step=min(e2e_ms, e2e_host_ms), graph_ms_per_step=e2e_ms, host_ms_per_step=e2e_host_ms,
                       serial_ms_per_step=e2e_serial_ms)
        if e2e_host_ms < e2e_ms:
            e2e_res["mode"] = ("host-launched pipeline (faster than its CUDA-graph capture on this run): step i+1's "
                               "copy-in and step i-1's copy-out overlap step i (two copy streams, double buffers); "
                               "every step copies its q/k/v in from pinned host memory and its attn_out back")

    cpu_line = None
    if cpu:
        import oracle  # checker / CPU baseline only

        oracle.build()
        val, desc = cpu_sample(torch, cache, q, k, v, dev, target_s=8.0, nthreads=1)
        cpu_line = {"value": val, "unit": UNIT, "cores": 1, "kind": "port (sampled, scaled)", "sample": desc}
    cache.close()
    # a graph that holds NCCL calls must be released before the process group
    if graph is not None:
        torch.cuda.synchronize(dev)
        graph.reset()
        del graph
    if e2e_res is not None:
        e2e_res.pop("graph", None)
    h2d = int((q.numel() + k.numel() + v.numel()) * 2)
    d2h = int((gathered if heads else out).numel() * 2)
    return dict(t_ms=t_ms, steps=steps, launches=launches, attend_ms=attend_ms, attend_launches=attend_launches,
                kv_count=kv_count, clocks=clocks, parity=parity, e2e=e2e_res, h2d=h2d, d2h=d2h, cpu=cpu_line,
                device_status=int(status), gather=gather if heads else None)


def measure_e2e(args, torch, sa, dev, stream, barrier, cache, cos, sin, q, k, v, out, gqa, heads, gathered, spg):
    """End to end: every step copies q/k/v in from pinned host memory and its attn_out back.

    Three loops, all timed with CUDA events on the compute stream:
      serial    copy-in, the operator, copy-out, one after the other (host launches);
      host      step i+1's copy-in (one stream) and step i-1's copy-out (another stream) overlap
                step i, double-buffered device inputs/outputs, launched from the host;
      graph     the same pipeline for S consecutive steps captured as one CUDA graph and replayed
                (the reported `e2e`; S divides the step count).
    """
    hq_ = q.cpu().pin_memory()
    hk_ = k.cpu().pin_memory()
    hv_ = v.cpu().pin_memory()
    res_t = gathered if heads else out
    hout = torch.empty_like(res_t, device="cpu").pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def serial_step():
        dq.copy_(hq_, non_blocking=True)
        dk.copy_(hk_, non_blocking=True)
        dv.copy_(hv_, non_blocking=True)
        hout.copy_(gqa(dq, dk, dv), non_blocking=True)

    for _ in range(3):
        serial_step()
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for _ in range(args.steps):
        serial_step()
    x1.record(stream)
    barrier()
    serial_ms = x0.elapsed_time(x1) / args.steps

    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(res_t))
            for _ in range(2)]
    houts = [torch.empty_like(res_t, device="cpu").pin_memory() for _ in range(2)]
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("ready", "done", "copied")}

    def pipeline(nsteps, cur):
        cs_in.wait_stream(cur)
        cs_out.wait_stream(cur)
        for i in range(nsteps):
            sl = i % 2
            dq_, dk_, dv_, do_ = bufs[sl]
            with torch.cuda.stream(cs_in):
                if i >= 2:
                    cs_in.wait_event(ev["done"][sl])  # step i-2 has read this slot's inputs
                dq_.copy_(hq_, non_blocking=True)
                dk_.copy_(hk_, non_blocking=True)
                dv_.copy_(hv_, non_blocking=True)
                ev["ready"][sl].record(cs_in)
            cur.wait_event(ev["ready"][sl])
            if i >= 2:
                cur.wait_event(ev["copied"][sl])  # step i-2's output has left this slot
            if heads:
                gqa(dq_, dk_, dv_, res_=do_)
            else:
                gqa(dq_, dk_, dv_, out_=do_)
            ev["done"][sl].record(cur)
            with torch.cuda.stream(cs_out):
                cs_out.wait_event(ev["done"][sl])
                houts[sl].copy_(do_, non_blocking=True)
                ev["copied"][sl].record(cs_out)
        cur.wait_stream(cs_in)
        cur.wait_stream(cs_out)

    pipeline(4, stream)
    barrier()
    x0.record(stream)
    pipeline(args.steps, stream)
    x1.record(stream)
    barrier()
    host_ms = x0.elapsed_time(x1) / args.steps

    # as many steps per graph as divide the step count (up to 50): the pipeline fills and drains
    # once per replay
    per_graph = next(s for s in (50, 40, 30, 25, 20, 10, 8, 6, 5, 4, 2, 1) if args.steps % s == 0 and s % spg == 0) \
        if args.steps % spg == 0 else None
    graph_ms, mode = host_ms, "host launches (the step count does not split into graph replays)"
    g = None
    if per_graph is not None and not args.no_graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            pipeline(per_graph, torch.cuda.current_stream(dev))
        for _ in range(2):
            g.replay()
        barrier()
        x0.record(stream)
        for _ in range(args.steps // per_graph):
            g.replay()
        x1.record(stream)
        barrier()
        graph_ms = x0.elapsed_time(x1) / args.steps
        mode = (f"CUDA graph of {per_graph} pipelined steps, replayed: step i+1's copy-in and step i-1's "
                f"copy-out overlap step i (two copy streams, double buffers); every step copies its q/k/v "
                f"in from pinned host memory and its attn_out back")
        torch.cuda.synchronize(dev)
        g.reset()
    return {"ms_per_step": graph_ms, "mode": mode, "host_ms_per_step": host_ms, "graph_ms_per_step": graph_ms,
            "serial_ms_per_step": serial_ms}


def decode_line(r, world, heads):
    """The JSON fields of one measured decode mode."""
    peak, peak_kind = load_peaks()
    kv_count = r["kv_count"]
    hq_local = kv_count * (HQ // HKV)
    rows_mult = 1 if heads else world  # sequences decoded per step = B * rows_mult
    abytes = attend_bytes(hkv=kv_count, hq=hq_local)  # this rank's share
    achieved = abytes / (r["attend_ms"] * 1e-3) / 1e9
    line = {
        "value": B * rows_mult / (r["t_ms"] * 1e-3), "ms_per_step": r["t_ms"], "steps": r["steps"],
        "gpu_launches": int(r["launches"]),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_PER_CALL if not heads else None,
                     "traffic_decode_stream": NCU_TRAFFIC_DECODE_STREAM if not heads else None,
                     "kernel": KERNEL_NOTE, "launches_per_call": r["attend_launches"],
                     "algorithmic_bytes": abytes, "ms_per_call": r["attend_ms"],
                     "peak_source": f"{peak_kind} hbm_gbs", "per": "rank"},
        "step_bytes": algorithmic_bytes(hkv=kv_count, hq=hq_local),  # per rank
        "step_gbs": algorithmic_bytes(hkv=kv_count, hq=hq_local) / (r["t_ms"] * 1e-3) / 1e9,
        "clocks": r["clocks"],
        "device_status": r["device_status"],
    }
    if r["e2e"] is not None:
        e = r["e2e"]
        line["e2e"] = {"value": B * rows_mult / (e["ms_per_step"] * 1e-3), "unit": UNIT,
                       "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                       "ms_per_step": e["ms_per_step"], "mode": e["mode"],
                       "host_launch_value": B * rows_mult / (e["host_ms_per_step"] * 1e-3),
                       "graph_value": B * rows_mult / (e["graph_ms_per_step"] * 1e-3),
                       "serial_value": B * rows_mult / (e["serial_ms_per_step"] * 1e-3),
                       "serial_ms_per_step": e["serial_ms_per_step"]}
    if r["parity"] is not None:
        line["parity_max_abs"] = r["parity"]["max_abs"]
        line["parity"] = r["parity"]
    return line


def run_gqa_decode(args):
    import torch
    import torch.distributed as dist

    import smallaios_b200 as sa
    from smallaios_b200._lib import lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    heads = args.mode == "heads" and world > 1
    r = measure_decode(args, torch, dist, sa, lib, dev, world, rank, local, heads=heads, gather=args.gather,
                       e2e=True, cpu=rank == 0 and world == 1 and not args.no_cpu_baseline)
    gather_desc = {"peer": "attn_out stored to every rank by the decode merge over NVLink, gather completed "
                           "on the device (epoch signals, bounded wait)",
                   "nccl": "NCCL all-gather of attn_out"}
    line = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong" if heads else "weak", "vs_baseline": None,
            "dtype": "int4-kv/bf16-act/f32-acc", "data": "synthetic (seeded normal, std 1.28)",
            "config": {"workload": WORKLOAD,
                       "batch_per_gpu": B if not heads else f"{B} (kv heads {r['kv_count']} of {HKV})",
                       "global_batch": B * (1 if heads else world), "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                       "context": T, "kv_bits": BITS, "rope_theta": THETA,
                       "parallelism": (f"kv-head-sharded x{world}, {gather_desc[args.gather]}" if heads
                                       else f"batch-sharded x{world} (no collective)"),
                       "l2": f"cache {2 * B * HKV * T * (CB + 8) / 1e6:.0f} MB > 126 MB L2 per step; no flush",
                       "launch": "host launches" if args.no_graph else
                       "CUDA graph of consecutive steps, replayed (launches linked by programmatic dependencies)"}}
    line.update(decode_line(r, world, heads))
    if r["cpu"] is not None:
        line["cpu_baseline"] = r["cpu"]
    if world > 1 and not heads and not args.no_heads:
        # The head-sharded mode on the same ranks: the same B sequences split by KV head, gathered.
        h = measure_decode(args, torch, dist, sa, lib, dev, world, rank, local, heads=True, gather=args.gather,
                           e2e=False, cpu=False)
        hl = decode_line(h, world, True)
        t1 = r["t_ms"]  # every rank of the batch mode runs the whole one-GPU step
        hl.update(gather=args.gather, gather_kind=gather_desc[args.gather], scaling="strong",
                  global_batch=B, kv_heads_per_rank=h["kv_count"],
                  efficiency_vs_1gpu=t1 / (world * h["t_ms"]),
                  note="efficiency_vs_1gpu = (this mode's tokens/s) / (N x one GPU's tokens/s on the whole "
                       "step); one GPU's step time is the batch mode's per-rank step")
        line["heads"] = hl
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
