"""Benchmark of the HOFA decode hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

One step = one HOFA decode step of the attention core for a batch of B
sequences on every GPU (d_model=1024 -> H=16, d_h=64,
r=16, cache length L=4096, bf16 activations, float32 GLA state), i.e. one
``hofa_decode_fwd`` launch per GPU: split-K softmax over the outlier cache,
GLA state update + readout, RMSNorm, blend.  Sequences are sharded across
GPUs with no collective (weak scaling); rank 0 prints one JSON line with the
whole-job tokens/s (device time, max over ranks).

* ``value``: steps timed with CUDA events on device-resident inputs.  The
  caches of consecutive steps rotate through enough independent sets to
  exceed 3x the L2 size, so every step streams its cache from HBM.
* ``e2e``: the same step through the C ABI (``hofa_decode_fwd`` with
  pre-packed arguments) with the step's inputs (new token q/k/v, log decay,
  mix gate) copied from pinned host memory and the output copied back and
  read on the host every step (CUDA runtime copies and a stream
  synchronisation per step); caches and GLA state stay resident in HBM (as
  in any decode loop) and rotate through the same sets as ``value``.
* ``roofline``: algorithmic HBM bytes of one launch
  (B*H*(L*(r+d_h)*2 + (d_h-r)*d_h*4*2)) / its average duration, against the
  measured copy bandwidth in MEASURED_PEAKS.json.
* ``cpu_baseline`` / ``--impl reference``: the reference's CPU computation of
  the same step (the oracle restatement of the training layer's decode core,
  src/HybridOutlierFactorizedAttentionTrain.py:403-436) in float32 on the
  host cores, timed on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "HOFA decode tokens/s (350M, B=1/4/64) & prefill tok/s; % of HBM/TC roofline"
H, D, R, L = 16, 64, 16, 4096
J = D - R
FALLBACK_HBM_GBS = 6650.0


def algorithmic_bytes(B: int) -> int:
    return B * H * (L * (R + D) * 2 + J * D * 4 * 2)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(B: int):
    """dram bytes (read + write) per launch from the committed ncu summary of
    this workload, if present (line ``traffic_bytes_per_launch_B<B>: N``)."""
    p = os.path.join(ROOT, "profiles", "hofa_decode_config1.md")
    if not os.path.exists(p):
        return None
    key = f"traffic_bytes_per_launch_B{B}:"
    for line in open(p):
        if line.strip().startswith(key):
            try:
                return int(line.split(":", 1)[1].strip().split()[0].replace(",", ""))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the GPU works."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        rows = [l for (ts, l) in self.lines if t0 - 0.06 <= ts <= t1 + 0.06] or [l for _, l in self.lines[-3:]]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in rows:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- inputs
def make_step_inputs(B, device, seed, dtype=torch.bfloat16):
    """Config-1 inputs: caches from N(0,1) projections, state ~ N(0, 0.1),
    log decay = logsigmoid(x.W_d)/16 and mix = sigmoid(x.W_m) for one new token."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(B, 1, 1024, generator=g)
    Wq, Wk, Wv = (torch.randn(1024, 1024, generator=g) * 0.02 for _ in range(3))
    Wd, Wm = torch.randn(1024, H, generator=g) * 0.02, torch.randn(1024, H, generator=g) * 0.02
    for h in range(H):
        Wq[h * D:h * D + R] *= 8
        Wk[h * D:h * D + R] *= 8
    sf = D ** 0.25
    q = (x @ Wq.T / sf).view(B, 1, H, D).transpose(1, 2)
    k = (x @ Wk.T / sf).view(B, 1, H, D).transpose(1, 2)
    v = (x @ Wv.T).view(B, 1, H, D).transpose(1, 2)
    log_gamma = (F.logsigmoid(x @ Wd) / 16).view(B, 1, H).transpose(1, 2)
    mix = torch.sigmoid(x @ Wm).view(B, 1, H).transpose(1, 2)
    return dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), log_gamma=log_gamma.float().contiguous(),
                mix=mix.to(dtype).contiguous(), norm_w=torch.ones(H, D), Wk=Wk, Wv=Wv)


KEY_STD = 8 * 0.02 * 1024 ** 0.5 / D ** 0.25   # outlier key channel of an N(0,1)-input projection
VAL_STD = 0.02 * 1024 ** 0.5                     # value channel of the same projection


def make_cache(B, device, seed, dtype=torch.bfloat16):
    """Synthetic caches with the per-channel statistics of config 1's
    N(0,1)-input projections (outlier keys std ~1.81, values std 0.64),
    drawn directly on the GPU so that set-up of many cache sets stays fast."""
    g = torch.Generator(device=device).manual_seed(seed)
    ck = (torch.randn(B, H, L, R, device=device, generator=g) * KEY_STD).to(dtype)
    cv = (torch.randn(B, H, L, D, device=device, generator=g) * VAL_STD).to(dtype)
    st = torch.randn(B, H, J, D, device=device, generator=g) * 0.1
    return ck, cv, st


# ----------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch.distributed as dist
    from outlierneuronattention_b200 import _capi
    from outlierneuronattention_b200.hofa_decode import decode_args, decode_workspace, fused_hofa_decode

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B = args.batch
    props = torch.cuda.get_device_properties(dev)
    l2 = props.L2_cache_size if hasattr(props, "L2_cache_size") else 126 * 2 ** 20
    per_set = algorithmic_bytes(B)
    nsets = max(2, math.ceil(3 * l2 / per_set))

    inp = make_step_inputs(B, dev, seed=1000 + rank)
    q, k, v = inp["q"].to(dev), inp["k"].to(dev), inp["v"].to(dev)
    lg, mix, nw = inp["log_gamma"].to(dev), inp["mix"].to(dev), inp["norm_w"].to(dev)
    sets = [make_cache(B, dev, seed=7 * rank + i) for i in range(nsets)]
    outs = [torch.empty(B, H, J, D, device=dev) for _ in range(nsets)]
    y = torch.empty_like(q)
    ws = decode_workspace(dev, B, H, D)
    split = args.split_k or 0
    fmt = _capi.FORMATS[_capi.DecodeArgs]
    bufs = [fmt.pack(*decode_args(q, k, v, ck, cv, st, outs[i], lg, mix, nw, R, L, 2.0, y, split_k=split,
                                  workspace=ws))
            for i, (ck, cv, st) in enumerate(sets)]
    fn = _capi.lib().hofa_decode_fwd

    stream = torch.cuda.Stream(dev)
    sh = stream.cuda_stream

    def launch_steps(n, start=0):
        for i in range(n):
            st = fn(bufs[(start + i) % nsets], sh)
            if st != 0:
                raise RuntimeError(_capi.lib().hofa_last_error().decode())

    # graph of `chunk` consecutive steps (removes host launch overhead)
    chunk = min(args.steps, 1000)
    with torch.cuda.stream(stream):
        launch_steps(nsets)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch_steps(chunk)
    torch.cuda.synchronize()

    def run(nsteps):
        full, rem = divmod(nsteps, chunk)
        for _ in range(full):
            graph.replay()
        if rem:
            launch_steps(rem)

    if args.profile:
        # small, self-contained command for ncu: the graph's steps only
        with torch.cuda.stream(stream):
            run(args.warmup)
            run(args.steps)
        torch.cuda.synchronize()
        print(json.dumps({"profile_run": True, "steps": args.steps, "batch": B, "nsets": nsets}))
        return

    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                           if "CUDA_VISIBLE_DEVICES" in os.environ else local)
    sampler.start()
    t_load0 = time.time()
    with torch.cuda.stream(stream):
        # warm-up: the requested steps, and at least ~0.4 s of work so clocks settle under load
        run(args.warmup)
        tw = time.time()
        while time.time() - tw < 0.4:
            run(chunk)
            stream.synchronize()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_timed0 = time.time()
        # an untimed lead-in replay keeps the GPU busy while e0 and the timed
        # graph launches are enqueued, so no host launch latency falls between
        # e0 and the first timed step
        run(chunk)
        e0.record(stream)
        run(args.steps)
        e1.record(stream)
        stream.synchronize()
        t_timed1 = time.time()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t_timed0 if t_timed1 - t_timed0 > 0.15 else t_load0, t_timed1)
    ms = e0.elapsed_time(e1)
    ms_t = torch.tensor([ms], device=dev)
    per_rank = [ms]
    if world > 1:
        all_ms = torch.empty(world, device=dev)
        dist.all_gather_into_tensor(all_ms, ms_t)
        per_rank = all_ms.tolist()
    ms_max = max(per_rank)
    ms_step = ms_max / args.steps
    value = B * world * args.steps / (ms_max / 1e3)

    # ---- e2e through the public operator with host buffers ----------------
    # The step's inputs (q, k, v, log_gamma, mix) sit in one pinned host buffer
    # at 256-byte aligned offsets and cross PCIe in one copy per step, as a
    # serving loop would stage them; the operator runs on views of the device
    # copy, and the step's output Y is read back to the host.
    parts = (("q", inp["q"]), ("k", inp["k"]), ("v", inp["v"]), ("lg", inp["log_gamma"]), ("mix", inp["mix"]))
    offs, nbytes = {}, 0
    for name, t in parts:
        offs[name] = nbytes
        nbytes += (t.numel() * t.element_size() + 255) // 256 * 256
    hstage = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dstage = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def view(buf, name, t):
        n = t.numel() * t.element_size()
        return buf[offs[name]:offs[name] + n].view(t.dtype).view(t.shape)

    for name, t in parts:
        view(hstage, name, t).copy_(t.cpu())
    dq, dk, dv, dlg, dmix = (view(dstage, name, t) for name, t in parts)
    yh = torch.empty(B, H, 1, D, dtype=q.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for _, t in parts)
    d2h = yh.numel() * yh.element_size()
    ck0, cv0, st0 = sets[0]
    e2e_steps = max(args.steps, 50)

    # The C ABI call a serving loop makes: hofa_decode_args packed once per
    # (cache, state direction) -- the GLA state ping-pongs between two
    # buffers -- and hofa_decode_fwd called with it every step; the steps walk
    # the same rotating cache sets as the device-timed loop, so every step
    # streams its cache from HBM.  The copies and the stream synchronisation
    # are the CUDA runtime's own calls (the runtime the library links), as a
    # C or C++ caller makes them, and Y is read from the pinned host buffer.
    import ctypes
    from outlierneuronattention_b200.hofa_decode import decode_args
    ye = torch.empty(B, H, 1, D, dtype=q.dtype, device=dev)
    fmt_e2e = _capi.FORMATS[_capi.DecodeArgs]
    packed = [[fmt_e2e.pack(*decode_args(dq, dk, dv, ck_, cv_, s_in, s_out, dlg, dmix, nw, R, L, 2.0, ye, split or None))
               for s_in, s_out in ((st_, outs[j]), (outs[j], st_))]
              for j, (ck_, cv_, st_) in enumerate(sets)]
    decode_fwd = _capi.lib().hofa_decode_fwd
    cudart = ctypes.CDLL("libcudart.so.12")
    memcpy_async = cudart.cudaMemcpyAsync
    memcpy_async.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    memcpy_async.restype = ctypes.c_int
    stream_sync = cudart.cudaStreamSynchronize
    stream_sync.argtypes = [ctypes.c_void_p]
    stream_sync.restype = ctypes.c_int
    cur = torch.cuda.current_stream(dev)
    cur_handle = cur.cuda_stream
    d_in, h_in, d_y, h_y = dstage.data_ptr(), hstage.data_ptr(), ye.data_ptr(), yh.data_ptr()
    y_bits = yh.view(torch.int16).numpy().reshape(-1)   # the pinned result, read on the host
    nsets_e2e = len(packed)

    def e2e_step(i):
        if memcpy_async(d_in, h_in, nbytes, 1, cur_handle) != 0:   # cudaMemcpyHostToDevice
            raise RuntimeError("cudaMemcpyAsync (inputs) failed")
        status = decode_fwd(packed[i % nsets_e2e][(i // nsets_e2e) % 2], cur_handle)
        if status != 0:
            raise RuntimeError(_capi.lib().hofa_last_error().decode())
        if memcpy_async(d_y, h_y, d2h, 2, cur_handle) != 0:        # cudaMemcpyDeviceToHost
            raise RuntimeError("cudaMemcpyAsync (Y) failed")
        if stream_sync(cur_handle) != 0:
            raise RuntimeError("cudaStreamSynchronize failed")
        return int(y_bits[0])

    for i in range(5):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = B * world * e2e_steps / e2e_t.item()

    # ---- roofline of the decode kernel (this arm's only kernel) ------------
    peak, peak_kind = peaks()
    achieved = algorithmic_bytes(B) / (ms_step / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": ncu_traffic(B), "algorithmic_bytes_per_launch": algorithmic_bytes(B)}

    out = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": f"config1-decode-B{B}-L{L}", "d_model": 1024, "heads": H, "d_head": D, "r": R,
                      "cache_len": L, "batch_per_gpu": B, "global_batch": B * world,
                      "split_k": split or int(_capi.lib().hofa_decode_choose_split(B, H, L, props.multi_processor_count)),
                      "l2": f"inputs larger than L2: {nsets} rotating cache sets x {per_set / 1e6:.1f} MB",
                      "parallelism": f"batch-sharded decode over {world} GPU(s), no collective"},
           "roofline": roofline,
           "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h,
                   "api": "C ABI hofa_decode_fwd with pre-packed hofa_decode_args (ctypes), one staged H2D copy "
                          "and the D2H copy of Y by cudaMemcpyAsync, cudaStreamSynchronize and a host read of Y every "
                          "step; rotating cache sets (no L2 reuse)"},
           "gpu_launches": args.steps, "clocks": clocks,
           "per_rank_us_per_step": [round(1e3 * m / args.steps, 3) for m in per_rank]}
    if not args.no_prefill:
        out["prefill"] = measure_prefill(dev)
    if not args.no_config4 and world == 1:
        out["config4"] = measure_config4(dev)
        out["layer_step"] = [measure_layer_step(dev, B=1), measure_layer_step(dev, B=4)]
        out["decode_batches"] = [measure_decode_batch(dev, 1), measure_decode_batch(dev, 64, steps=50)]
    if not args.no_config4 and world > 1:
        sp = measure_seqpar(dev, world)
        out["config4_seqpar"] = sp.pop("summary")
        out["decode_head_sharded"] = [measure_decode_head_sharded(dev, world, B=1),
                                      measure_config4_decode_head_sharded(dev, world, sp)]
    if not args.no_config3:
        out["config3"] = measure_config3(dev, world, rank)
    if not args.no_triton_reference and world == 1:
        out["triton_reference"] = measure_triton_reference(dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(B, args.cpu_seconds)
        out["cpu_baseline"]["reference_layer"] = cpu_reference_layer(B, args.cpu_seconds / 2)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------- prefill
def measure_prefill(dev, B=4, T=8192, steps=5, warmup=3, name="config2"):
    """BASELINE config 2 prefill of the attention core (bf16, B=4, T=8192,
    H=16, d_h=64, r=16): gates + RoPE + cache export (hofa_prep_fwd), the
    chunked GLA (hofa_prefill_gla_fwd) and the tcgen05 outlier attention
    (hofa_prefill_outlier_fwd), on projections already in HBM.  Inputs
    (3 x 64 MiB) exceed L2.  Each operator is timed with CUDA events over
    `steps` back-to-back calls (the host enqueues ahead of the GPU, so no
    host time falls inside the interval), after `warmup` untimed calls; a
    write of 2 x L2 between the operators evicts what the previous one left
    in L2.  prep rotates q and k in place, so its repeated calls rotate
    already-rotated rows: the same work and bytes, other values."""
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    from outlierneuronattention_b200.exact_attention import exact_attention_triton
    from outlierneuronattention_b200.modules import RotaryEmbedding
    from outlierneuronattention_b200.prep import prep
    g = torch.Generator(device=dev).manual_seed(3)
    x3 = torch.randn(B, T, 3, H, D, device=dev, generator=g).to(torch.bfloat16)
    q0, k0, v = (x3[:, :, i].transpose(1, 2) for i in range(3))  # [B,H,T,D] views, as the layer's projections
    gate_w = torch.randn(H, 2 * D, device=dev, generator=g) * 0.1
    gate_b = torch.full((H,), -1.0, device=dev)
    mix_w = torch.randn(H, 2 * D, device=dev, generator=g) * 0.1
    mix_b = torch.zeros(H, device=dev)
    rope = RotaryEmbedding(R).to(dev)
    gs = torch.ones(1, H, 1, D, device=dev)
    q, k = q0.clone(), k0.clone()
    lg = torch.empty(B, H, T, device=dev)
    mix = torch.empty(B, H, T, device=dev, dtype=torch.bfloat16)
    ck = torch.empty(B, H, T, R, device=dev, dtype=torch.bfloat16)
    cv = torch.empty(B, H, T, D, device=dev, dtype=torch.bfloat16)
    y = torch.empty(B, H, T, D, device=dev, dtype=torch.bfloat16)
    st = torch.empty(B, H, J, D, device=dev)
    flush = torch.empty(2 * 126 * 2 ** 20 // 4, device=dev)
    # the reference model's per-channel decay variant (learnable_alpha), timed
    # on its own: not part of the prefill total
    la = torch.randn(1, H, 1, J, device=dev, generator=g) * 0.5
    ops = {
        "prep": lambda: prep(q, k, v, gate_w, gate_b, lg, mix_w=mix_w, mix_b=mix_b, mix_out=mix,
                             cos=rope.cos_cached, sin=rope.sin_cached, R=R, pos0=0, cache_k=ck, cache_v=cv),
        "gla": lambda: gla_forward(q, k, v, lg, R, mix_g=mix, gla_scale=gs, y=y, state_out=st),
        "outlier": lambda: exact_attention_triton(q, k, v, R, 2.0, mix, out=y),
        "gla_per_channel_decay": lambda: gla_forward(q, k, v, lg, R, log_alpha=la, mix_g=mix, gla_scale=gs,
                                                     y=y, state_out=st),
    }
    ms = {}
    for name_, fn in ops.items():
        for _ in range(warmup):
            fn()
        flush.zero_()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms[name_] = e0.elapsed_time(e1) / steps
    total = ms["prep"] + ms["gla"] + ms["outlier"]
    attn_flops = B * H * (R + D) * T * T            # causal QK^T + PV, 2 flops per MAC
    gla_flops = 6 * B * H * J * D * T
    bf16_peak, hbm_peak = 1647.9, 6650.0
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
        bf16_peak, hbm_peak = float(peaks["bf16_tflops"]), float(peaks["hbm_gbs"])
    ach = attn_flops / (ms["outlier"] / 1e3) / 1e12
    # GLA algorithmic bytes: Q_I and K_I as read (32-byte sectors of their 48-channel rows: 3/4 of each
    # 128-byte row), V, log decay and blend (fp32 / bf16), y written
    gla_bytes = B * H * T * (2 * (D * 2 * 3 // 4) + D * 2 + 4 + 2 + D * 2)
    gla_ach = gla_bytes / (ms["gla"] / 1e3) / 1e9
    return {"workload": f"{name}-prefill-B{B}-T{T}", "tokens_per_s": round(B * T / (total / 1e3), 1),
            "ms": round(total, 4), "ms_by_kernel": {k_: round(v_, 4) for k_, v_ in ms.items()},
            "timing": f"CUDA events over {steps} back-to-back calls per operator, inputs larger than L2",
            "algorithmic_flops": attn_flops + gla_flops, "exps": B * H * T * T // 2,
            "roofline_outlier_kernel": {"bound": "tensor", "achieved": round(ach, 2), "peak": bf16_peak,
                                        "unit": "TFLOP/s", "frac": round(ach / bf16_peak, 4),
                                        "peak_source": "measured bf16_tflops (burst)"},
            "roofline_gla_kernel": {"bound": "hbm", "achieved": round(gla_ach, 1), "peak": hbm_peak, "unit": "GB/s",
                                    "frac": round(gla_ach / hbm_peak, 4), "algorithmic_bytes": gla_bytes,
                                    "peak_source": "measured hbm_gbs"},
            "gla_per_channel_decay_ms": round(ms["gla_per_channel_decay"], 4)}


def measure_decode_batch(dev, B, steps=200, reps=3):
    """Config-1 decode (L=4096, H=16, d_h=64, r=16, bf16) at another batch size:
    `hofa_decode_fwd` steps replayed from a CUDA graph over rotating cache
    sets of at least 3 x L2 (every step streams its cache from HBM), timed
    with CUDA events; tokens/s and the HBM roofline of the step."""
    from outlierneuronattention_b200 import _capi
    from outlierneuronattention_b200.hofa_decode import decode_args, decode_workspace
    per_set = algorithmic_bytes(B)
    nsets = max(2, math.ceil(3 * 126 * 2 ** 20 / per_set))
    inp = make_step_inputs(B, "cpu", seed=5000 + B)
    q, k, v = (inp[n].to(dev) for n in ("q", "k", "v"))
    lg, mix, nw = inp["log_gamma"].to(dev), inp["mix"].to(dev), inp["norm_w"].to(dev)
    sets = [make_cache(B, dev, seed=100 * B + i) for i in range(nsets)]
    outs = [torch.empty(B, H, J, D, device=dev) for _ in range(nsets)]
    y = torch.empty_like(q)
    ws = decode_workspace(dev, B, H, D)
    fmt = _capi.FORMATS[_capi.DecodeArgs]
    bufs = [fmt.pack(*decode_args(q, k, v, ck, cv, st, outs[i], lg, mix, nw, R, L, 2.0, y, workspace=ws))
            for i, (ck, cv, st) in enumerate(sets)]
    fn = _capi.lib().hofa_decode_fwd
    stream = torch.cuda.Stream(dev)

    def launch(n):
        for i in range(n):
            if fn(bufs[i % nsets], stream.cuda_stream) != 0:
                raise RuntimeError(_capi.lib().hofa_last_error().decode())

    with torch.cuda.stream(stream):
        launch(nsets)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch(steps)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * steps)
    del graph
    peak, kind = peaks()
    ach = per_set / (us / 1e6) / 1e9
    split = int(_capi.lib().hofa_decode_choose_split(B, H, L, torch.cuda.get_device_properties(dev).multi_processor_count))
    return {"workload": f"config1-decode-B{B}-L{L}", "us_per_step": round(us, 3), "tokens_per_s": round(B / (us / 1e6), 1),
            "algorithmic_bytes_per_step": per_set, "split_k": split, "rotating_sets": nsets,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_source": f"{kind} hbm_gbs"}}


def measure_config4(dev, steps=64, reps=3):
    """BASELINE config 4 on one GPU: the attention core's prefill at B=1,
    T=65536, and decode steps against a 65,600-token cache (B=1; two rotating
    168 MB cache sets, so every step streams its cache from HBM; the steps are
    replayed from a CUDA graph and timed with CUDA events)."""
    from outlierneuronattention_b200 import _capi, fused_hofa_decode
    out = {"workload": "config4-B1-T65536", "prefill": measure_prefill(dev, B=1, T=65536, steps=3, warmup=1,
                                                                       name="config4")}
    L4, B4 = 65600, 1
    g = torch.Generator(device=dev).manual_seed(11)
    sets = []
    for _ in range(2):
        ck = (torch.randn(B4, H, L4, R, device=dev, generator=g) * KEY_STD).to(torch.bfloat16)
        cv = (torch.randn(B4, H, L4, D, device=dev, generator=g) * VAL_STD).to(torch.bfloat16)
        sets.append((ck, cv))
    inp = make_step_inputs(B4, "cpu", seed=4000)
    q, k, v = (inp[n].to(dev) for n in ("q", "k", "v"))
    lg, mix, nw = inp["log_gamma"].to(dev), inp["mix"].to(dev), inp["norm_w"].to(dev)
    st = [torch.randn(B4, H, J, D, device=dev, generator=g) * 0.1, torch.empty(B4, H, J, D, device=dev)]

    def launch(n):
        for i in range(n):
            ck, cv = sets[i % 2]
            fused_hofa_decode(q, k, v, ck, cv, st[i % 2], st[(i + 1) % 2], lg, mix, nw, R, L4, 2.0)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        launch(4)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch(steps)
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * steps)
    del graph
    nbytes = B4 * H * (L4 * (R + D) * 2 + J * D * 4 * 2)
    peak, kind = peaks()
    ach = nbytes / (us / 1e6) / 1e9
    out["decode"] = {"batch": B4, "cache_len": L4, "us_per_step": round(us, 3),
                     "tokens_per_s": round(B4 / (us / 1e6), 1), "algorithmic_bytes_per_step": nbytes,
                     "split_k": int(_capi.lib().hofa_decode_choose_split(B4, H, L4, torch.cuda.get_device_properties(dev).multi_processor_count)),
                     "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(ach / peak, 4), "peak_source": f"{kind} hbm_gbs"}}
    return out


def measure_seqpar(dev, world, steps=3, warmup=2):
    """BASELINE config 4 prefill of the attention core (B=1, T=65536)
    sequence-sharded over the ranks (zig-zag blocks; two batched GLA passes
    around the block-state exchange, outlier attention against the key prefix
    that NCCL point-to-point transfers fill in during the GLA passes).  Every
    rank draws the same whole-sequence inputs and takes its two blocks; the
    time per prefill is the max over ranks of CUDA-event times around the
    whole sharded core, exchange included, with a per-phase breakdown (median
    over the timed runs, max over ranks).  After timing, each rank checks its
    output rows and the final GLA state against a one-GPU run of the same
    operators over the whole sequence (``parity_maxabs``, max over ranks)."""
    import torch.distributed as dist
    from outlierneuronattention_b200 import seqpar
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    from outlierneuronattention_b200.exact_attention import exact_attention_triton
    B4, T4 = 1, 65536
    rank = dist.get_rank()
    g = torch.Generator(device=dev).manual_seed(21)
    x3 = torch.randn(B4, T4, 3, H, D, device=dev, generator=g).to(torch.bfloat16)
    qf, kf, vf = (x3[:, :, i].transpose(1, 2) for i in range(3))
    lgf = torch.nn.functional.logsigmoid(torch.randn(B4, H, T4, device=dev, generator=g) + 2.0) / 16
    mixf = torch.sigmoid(torch.randn(B4, H, T4, device=dev, generator=g)).to(torch.bfloat16)
    take = lambda x: seqpar.shard_tokens(x, world, rank, dim=2).contiguous()
    q, k, v, lg, mix = take(qf), take(kf), take(vf), take(lgf), take(mixf)
    gs = torch.ones(1, H, 1, D, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times, phases = [], []
    for it in range(warmup + steps):
        dist.barrier()
        torch.cuda.synchronize()
        timer = seqpar.PhaseTimer()
        e0.record()
        Y, S_end = seqpar.sharded_attention_core(q, k, v, lg, mix, R, 2.0, gs, T4, timer=timer)
        e1.record()
        torch.cuda.synchronize()
        if it >= warmup:
            times.append(e0.elapsed_time(e1))
            phases.append(timer.ms())
    names = list(phases[0].keys())
    ph = torch.tensor([statistics.median(p[n] for p in phases) for n in names] + [statistics.median(times)],
                      device=dev)
    dist.all_reduce(ph, op=dist.ReduceOp.MAX)
    ms = ph[-1].item()
    # parity: the same computation over the whole sequence on one GPU, in bf16
    # and in float32 (the float32 operators of this library on the same
    # bf16-valued inputs); the bf16 paths differ from each other in rounding
    # order (GLA output and attention term rounded separately here, the
    # attention term added into the rounded GLA output there)
    Yf = torch.empty(B4, H, T4, D, device=dev, dtype=torch.bfloat16)
    Sf = torch.empty(B4, H, J, D, device=dev)
    gla_forward(qf, kf, vf, lgf, R, mix_g=mixf, gla_scale=gs, y=Yf, state_out=Sf)
    exact_attention_triton(qf, kf, vf, R, 2.0, mixf, out=Yf)
    q32, k32, v32 = qf.float(), kf.float(), vf.float()
    Y32 = torch.empty(B4, H, T4, D, device=dev)
    S32 = torch.empty(B4, H, J, D, device=dev)
    gla_forward(q32, k32, v32, lgf, R, mix_g=mixf.float(), gla_scale=gs, y=Y32, state_out=S32)
    exact_attention_triton(q32, k32, v32, R, 2.0, mixf.float(), out=Y32)
    Y32l = take(Y32)
    err = torch.tensor([(Y.float() - Y32l).abs().max().item(), (take(Yf).float() - Y32l).abs().max().item(),
                        (Y.float() - take(Yf).float()).abs().max().item(), (S_end - S32).abs().max().item(),
                        (S_end - Sf).abs().max().item()], device=dev)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    del q32, k32, v32, Y32, Y32l
    summary = {"workload": f"config4-prefill-seqpar-B{B4}-T{T4}", "ranks": world, "ms": round(ms, 4),
               "tokens_per_s": round(B4 * T4 / (ms / 1e3), 1),
               "phase_ms_max_over_ranks": {n: round(ph[i].item(), 4) for i, n in enumerate(names)},
               "parity_maxabs": {"y_vs_fp32": err[0].item(), "y_one_gpu_bf16_vs_fp32": err[1].item(),
                                 "y_vs_one_gpu_bf16": err[2].item(), "final_state_vs_fp32": err[3].item(),
                                 "final_state_vs_one_gpu_bf16": err[4].item(),
                                 "against": "the whole sequence on one GPU: float32 operators on the same "
                                            "bf16-valued inputs, and the bf16 operators"},
               "sharding": f"zig-zag: {2 * world} blocks of {T4 // (2 * world)} tokens, rank r owns r and {2 * world - 1}-r",
               "exchange": "K_O|V blocks into one token-major full-sequence buffer: in-place all_gather of the "
                           "first-half blocks, NCCL isend/irecv of the second-half blocks (during the first GLA "
                           "pass); all_gather of the GLA block states (under the attention)",
               "timed": "pack + GLA pass 1 + exchange + outlier attention (2 side streams) with the state "
                        "exchange and GLA pass 2 underneath + final add, max over ranks"}
    del x3, Yf
    return {"summary": summary, "q": q, "k": k, "v": v, "S_end": S_end, "kf": kf, "vf": vf, "T": T4}


def _decode_graph_time(launch, nsteps, reps, stream):
    """CUDA-event time per step of `nsteps` launches captured in one graph,
    replayed `reps` times behind an untimed lead-in replay."""
    with torch.cuda.stream(stream):
        launch()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch()
        graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        graph.replay()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * nsteps)
    del graph
    return us


def measure_decode_head_sharded(dev, world, B=1, steps=200, reps=3):
    """Config-1 decode (L=4096) with the heads split over the ranks: rank g
    runs the attention core of heads [16g/N, 16(g+1)/N) for all B sequences
    (no collective).  One decode step of the B sequences uses all N GPUs, so
    tokens/s = B / (max over ranks of the step time); each rank streams the
    caches of its heads from HBM (rotating sets larger than 3 x L2)."""
    import torch.distributed as dist
    from outlierneuronattention_b200 import _capi
    from outlierneuronattention_b200.hofa_decode import decode_args, decode_workspace
    from outlierneuronattention_b200.seqpar import head_range
    rank = dist.get_rank()
    h0, h1 = head_range(H, world, rank)
    Hg = h1 - h0
    per_set = B * Hg * (L * (R + D) * 2 + J * D * 4 * 2)
    nsets = max(2, math.ceil(3 * 126 * 2 ** 20 / per_set))
    inp = make_step_inputs(B, "cpu", seed=6000 + B)
    q, k, v = (inp[n][:, h0:h1].contiguous().to(dev) for n in ("q", "k", "v"))
    lg, mix = inp["log_gamma"][:, h0:h1].contiguous().to(dev), inp["mix"][:, h0:h1].contiguous().to(dev)
    nw = inp["norm_w"][h0:h1].contiguous().to(dev)
    sets = [[t[:, h0:h1].contiguous() for t in make_cache(B, dev, seed=300 + i)] for i in range(nsets)]
    outs = [torch.empty(B, Hg, J, D, device=dev) for _ in range(nsets)]
    y = torch.empty_like(q)
    ws = decode_workspace(dev, B, Hg, D)
    fmt = _capi.FORMATS[_capi.DecodeArgs]
    bufs = [fmt.pack(*decode_args(q, k, v, ck, cv, st, outs[i], lg, mix, nw, R, L, 2.0, y, workspace=ws))
            for i, (ck, cv, st) in enumerate(sets)]
    fn = _capi.lib().hofa_decode_fwd
    stream = torch.cuda.Stream(dev)

    def launch():
        for i in range(steps):
            if fn(bufs[i % nsets], stream.cuda_stream) != 0:
                raise RuntimeError(_capi.lib().hofa_last_error().decode())

    dist.barrier()
    us = _decode_graph_time(launch, steps, reps, stream)
    t = torch.tensor([us], device=dev)
    all_us = torch.empty(world, device=dev)
    dist.all_gather_into_tensor(all_us, t)
    us_max = all_us.max().item()
    peak, kind = peaks()
    ach = per_set / (us_max / 1e6) / 1e9
    split = int(_capi.lib().hofa_decode_choose_split(B, Hg, L, torch.cuda.get_device_properties(dev).multi_processor_count))
    return {"workload": f"config1-decode-B{B}-L{L}-head-sharded", "ranks": world, "heads_per_rank": Hg,
            "us_per_step": round(us_max, 3), "per_rank_us_per_step": [round(x, 3) for x in all_us.tolist()],
            "tokens_per_s": round(B / (us_max / 1e6), 1), "split_k": split,
            "per_rank_bytes_per_step": per_set,
            "per_rank_roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(ach / peak, 4), "peak_source": f"{kind} hbm_gbs"}}


def measure_config4_decode_head_sharded(dev, world, sp, nsteps=128, reps=3):
    """Config 4 after the sequence-sharded prefill: the outlier caches and GLA
    state are re-laid out from sequence shards to head shards (one
    all_to_all_single, timed), then 128 split-K decode steps over the 64k
    cache (rows T .. T+127 attended as the steps advance) run head-sharded,
    replayed from a CUDA graph.  Parity: each rank's first decode step against
    the same step over all heads with the whole-sequence caches."""
    import torch.distributed as dist
    from outlierneuronattention_b200 import _capi, fused_hofa_decode
    from outlierneuronattention_b200.seqpar import head_range, relayout_seq_to_head
    rank = dist.get_rank()
    T4 = sp["T"]
    cap = T4 + nsteps
    h0, h1 = head_range(H, world, rank)
    Hg = h1 - h0
    # one untimed call first: the first all_to_all of a process group sets up NCCL's connections
    relayout_seq_to_head(sp["k"][..., :R], sp["v"], sp["S_end"], T4, cap)
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ck, cv, st0 = relayout_seq_to_head(sp["k"][..., :R], sp["v"], sp["S_end"], T4, cap)
    e1.record()
    torch.cuda.synchronize()
    relayout_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(relayout_ms, op=dist.ReduceOp.MAX)
    g = torch.Generator(device=dev).manual_seed(31)
    newk = torch.randn(1, H, nsteps, R, device=dev, generator=g).to(torch.bfloat16)
    newv = torch.randn(1, H, nsteps, D, device=dev, generator=g).to(torch.bfloat16)
    ck[:, :, T4:] = newk[:, h0:h1]
    cv[:, :, T4:] = newv[:, h0:h1]
    inp = make_step_inputs(1, "cpu", seed=4100)
    q, k, v = (inp[n].to(dev) for n in ("q", "k", "v"))
    lg, mix, nw = inp["log_gamma"].to(dev), inp["mix"].to(dev), inp["norm_w"].to(dev)
    sl = lambda t: t[:, h0:h1].contiguous()
    qg, kg, vg, lgg, mixg, nwg = sl(q), sl(k), sl(v), sl(lg), sl(mix), nw[h0:h1].contiguous()
    st = [st0.clone(), torch.empty_like(st0)]
    ys = [torch.empty_like(qg) for _ in range(nsteps)]
    # parity: step 0 (T4 + 1 rows) over the head shard vs all heads with the whole-sequence caches
    y0 = fused_hofa_decode(qg, kg, vg, ck, cv, st[0], st[1], lgg, mixg, nwg, R, T4 + 1, 2.0)
    ckf = torch.cat([sp["kf"][..., :R], newk[:, :, :1]], dim=2).contiguous()
    cvf = torch.cat([sp["vf"], newv[:, :, :1]], dim=2).contiguous()
    sf = torch.empty(1, H, J, D, device=dev)
    S_full = torch.empty_like(sf)
    # the whole-sequence state of every head: gather the head shards (every rank has all of S_end anyway)
    S_full.copy_(sp["S_end"])
    yf = fused_hofa_decode(q, k, v, ckf, cvf, S_full, sf, lg, mix, nw, R, T4 + 1, 2.0)
    torch.cuda.synchronize()
    perr = torch.tensor([(y0.float() - yf[:, h0:h1].float()).abs().max().item(),
                         (st[1] - sf[:, h0:h1]).abs().max().item()], device=dev)
    dist.all_reduce(perr, op=dist.ReduceOp.MAX)
    del ckf, cvf

    def launch():
        for i in range(nsteps):
            fused_hofa_decode(qg, kg, vg, ck, cv, st[i % 2], st[(i + 1) % 2], lgg, mixg, nwg, R, T4 + 1 + i, 2.0)

    stream = torch.cuda.Stream(dev)
    dist.barrier()
    us = _decode_graph_time(launch, nsteps, reps, stream)
    t = torch.tensor([us], device=dev)
    all_us = torch.empty(world, device=dev)
    dist.all_gather_into_tensor(all_us, t)
    us_max = all_us.max().item()
    per_rank_bytes = Hg * ((T4 + nsteps // 2) * (R + D) * 2 + J * D * 4 * 2)
    peak, kind = peaks()
    ach = per_rank_bytes / (us_max / 1e6) / 1e9
    return {"workload": f"config4-decode-B1-L{T4}+{nsteps}-head-sharded", "ranks": world, "heads_per_rank": Hg,
            "relayout_ms": round(relayout_ms.item(), 4),
            "us_per_step": round(us_max, 3), "per_rank_us_per_step": [round(x, 3) for x in all_us.tolist()],
            "tokens_per_s": round(1 / (us_max / 1e6), 1), "decode_steps": nsteps,
            "parity_maxabs": {"y": perr[0].item(), "state": perr[1].item(),
                              "against": "the same decode step over all heads with the whole-sequence caches"},
            "per_rank_roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(ach / peak, 4), "peak_source": f"{kind} hbm_gbs",
                                  "bytes_per_step": per_rank_bytes}}


def measure_layer_step(dev, B=4, steps=64, reps=5):
    """Layer-level decode step (the drop-in module's forward_step with a
    pre-allocated cache of L=4096 rows, d_model=1024, H=16, r=16, bf16
    weights): the QKV projection, the fused decode step (hofa_decode_step_fwd:
    gates, RoPE, cache append and the attention core in one launch) and the
    output projection, replayed from a CUDA graph."""
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(0)
    cfg = ModelConfig(d_model=1024, num_heads=H, num_layers=1, r=R, chunk_size=64)
    m = HybridOutlierFactorizedAttention(cfg).to(device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(B, 1, 1024, device=dev, generator=g).to(torch.bfloat16)
    # 4 rotating caches (4 x 42 MB at B=4 > L2), so each step streams its cache from HBM
    caches = [((torch.randn(B, H, L, R, device=dev, generator=g) * KEY_STD).to(torch.bfloat16),
               (torch.randn(B, H, L, D, device=dev, generator=g) * VAL_STD).to(torch.bfloat16)) for _ in range(4)]
    st = (torch.randn(B, H, J, D, device=dev, generator=g) * 0.1, torch.empty(B, H, J, D, device=dev))

    def launch():
        for i in range(steps):
            m.forward_step(x, caches[i % 4], st, cache_seq_len=L - 1)

    with torch.no_grad():
        us = _decode_graph_time(launch, steps, reps, torch.cuda.Stream(dev))
    return {"workload": f"config1-layer-forward_step-B{B}-L{L}", "d_model": 1024, "us_per_step": round(us, 3),
            "tokens_per_s": round(B / (us / 1e6), 1),
            "note": "QKV projection (cuBLAS) + fused decode step + out_proj per step, CUDA graph"}


# ----------------------------------------------------------------------------- config 3: the 350M LM
def measure_config3(dev, world, rank, batches=(1, 4, 64), prompt=16384, new=256):
    """the 350M-shaped LM (24 layers, d_model 1024, 16
    heads of 64, r = 16, SwiGLU 4096, RMSNorm, vocabulary 32000, tied
    embedding, random init std 0.02, bf16) decodes `new` tokens greedily after
    a `prompt`-token prompt of uniform random token ids (seed 1), from one
    CUDA graph of two decode steps with the position and the sampling on the
    device (``lm.DecodeEngine``).  A batch that splits evenly over the ranks
    is batch-sharded (each rank prefills and decodes B/N sequences); smaller
    ones run as independent replicas.  Device time of the whole generation
    (CUDA events, max over ranks, after one untimed generation); the prompt's
    prefill runs once per batch, outside the timed region.  Roofline: weights
    plus every layer's outlier cache at the mean decode length, per step."""
    import torch.distributed as dist
    from outlierneuronattention_b200.lm import DecodeEngine, HofaLM, LMConfig
    cfg = LMConfig()
    torch.manual_seed(0)
    model = HofaLM(cfg).to(device=dev, dtype=torch.bfloat16).eval()
    nparam = model.num_parameters()
    peak, kind = peaks()
    rows = []
    for Bg in batches:
        shard = world > 1 and Bg >= world and Bg % world == 0
        B = Bg // world if shard else Bg
        g = torch.Generator().manual_seed(1 + (rank if (shard or world > 1) else 0))
        idx = torch.randint(0, cfg.vocab_size, (B, prompt), generator=g).to(dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logits0, caches, states = model.prefill(idx, prompt + new, batch_chunk=8)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        eng = DecodeEngine(model, caches, states, logits0, prompt)
        eng.capture(new)
        eng.generate(new)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        toks = eng.generate(new)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = ms.item()
        total = (Bg if shard else B * world) * new
        per_step_bytes = nparam * 2 + B * cfg.num_layers * cfg.num_heads * (
            (prompt + new // 2) * (cfg.r + 64) * 2 + (64 - cfg.r) * 64 * 4 * 2)
        bound = B / (per_step_bytes / (peak * 1e9))
        tps = total / (ms / 1e3)
        rows.append({"batch": Bg, "mode": ("batch-sharded" if shard else ("replicas" if world > 1 else "one GPU")),
                     "batch_per_rank": B, "tokens": total, "ms": round(ms, 3), "tokens_per_s": round(tps, 1),
                     "us_per_step": round(1e3 * ms / new, 2), "prefill_s": round(prefill_s, 3),
                     "hbm_bytes_per_step_per_rank": per_step_bytes,
                     "roofline": {"bound": "hbm", "tokens_per_s_bound_per_rank": round(bound, 1),
                                  "frac": round((tps / (total / new / B)) / bound, 4),
                                  "peak_source": f"{kind} hbm_gbs"},
                     "first_tokens": toks[0, :4].tolist()})
        eng.release()
        del eng, caches, states, logits0, toks
        torch.cuda.empty_cache()
    return {"workload": f"config3-350M-LM-decode-{new}-after-{prompt}", "params": nparam,
            "model": "24 x (RMSNorm, HOFA layer, RMSNorm, SwiGLU 4096), vocab 32000, tied embedding, bf16, random init",
            "sampling": "greedy, in the CUDA graph", "timing": "CUDA events around the graph replays, max over ranks",
            "rows": rows}


# ----------------------------------------------------------------------------- reference's Triton kernels
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _event_ms(fn, n, flush=None):
    """Mean CUDA-event time of `n` back-to-back calls (after a flush of L2)."""
    if flush is not None:
        flush.zero_()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def measure_triton_reference(dev):
    """The reference's own GPU implementation of the hot path -- its Triton
    kernels ``fused_hofa_decode`` (src/hofa_decode_triton.py:342),
    ``chunk_gla_inlier_fwd`` (src/chunk_gla_inlier.py:153) and
    ``exact_attention_triton`` (src/exact_attention.py:163), and its layer
    ``HybridOutlierFactorizedAttention`` -- imported unmodified from
    baseline/_ref (an install of the reference package) and run on this GPU
    with the same inputs, shapes and timing method as this library's arm:
    decode steps replayed from a CUDA graph over rotating cache sets larger
    than L2, prefill operators over back-to-back calls after an L2 flush.
    ``maxabs_vs_ours`` is the largest difference between the reference's
    outputs and this library's on the same inputs."""
    if not os.path.isdir(os.path.join(REF_DIR, "src")):
        return {"unavailable": "baseline/_ref is not installed"}
    sys.path.insert(0, REF_DIR)
    try:
        from src.chunk_gla_inlier import chunk_gla_inlier_fwd as ref_gla
        from src.exact_attention import exact_attention_triton as ref_attn
        from src.hofa_decode_triton import fused_hofa_decode as ref_decode
        from src.HybridOutlierFactorizedAttention import HybridOutlierFactorizedAttention as RefLayer
        from src.config import ModelConfig as RefConfig
    except Exception as e:  # noqa: BLE001
        sys.path.remove(REF_DIR)
        return {"unavailable": f"import of the reference failed: {e!r}"}
    from outlierneuronattention_b200 import (HybridOutlierFactorizedAttention, ModelConfig, exact_attention_triton,
                                             fused_hofa_decode)
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    out = {"source": "baseline/_ref (reference package, unmodified), Triton " + __import__("triton").__version__}
    try:
        # ---- decode, config 1 (B = 1, 4, 64) and config 4 ------------------------------------
        dec = []
        for B, steps in ((1, 200), (4, 200), (64, 20)):
            per_set = algorithmic_bytes(B)
            nsets = max(2, math.ceil(3 * 126 * 2 ** 20 / per_set))
            inp = make_step_inputs(B, "cpu", seed=7000 + B)
            q, k, v = (inp[n].to(dev) for n in ("q", "k", "v"))
            lg, mix, nw = inp["log_gamma"].to(dev), inp["mix"].to(dev), inp["norm_w"].to(dev)
            sets = [make_cache(B, dev, seed=500 * B + i) for i in range(nsets)]
            outs = [torch.empty(B, H, J, D, device=dev) for _ in range(nsets)]
            row = {"workload": f"config1-decode-B{B}-L{L}"}
            if B == 4:
                ck, cv, st = sets[0]
                s_ref, s_our = torch.empty_like(st), torch.empty_like(st)
                y_ref = ref_decode(q, k, v, ck, cv, st, s_ref, lg, mix, nw, R, L, 2.0)
                y_our = fused_hofa_decode(q, k, v, ck, cv, st, s_our, lg, mix, nw, R, L, 2.0)
                torch.cuda.synchronize()
                row["maxabs_vs_ours"] = {"y": (y_ref.float() - y_our.float()).abs().max().item(),
                                         "state": (s_ref - s_our).abs().max().item()}

            def launch(B=B, sets=sets, outs=outs, q=q, k=k, v=v, lg=lg, mix=mix, nw=nw, steps=steps, nsets=nsets):
                for i in range(steps):
                    ck, cv, st = sets[i % nsets]
                    ref_decode(q, k, v, ck, cv, st, outs[i % nsets], lg, mix, nw, R, L, 2.0)

            us = _decode_graph_time(launch, steps, 3, torch.cuda.Stream(dev))
            row.update({"us_per_step": round(us, 3), "tokens_per_s": round(B / (us / 1e6), 1),
                        "hbm_frac": round(per_set / (us / 1e6) / 1e9 / peaks()[0], 4)})
            dec.append(row)
            del sets, outs
        out["decode"] = dec
        # ---- prefill operators, config 2 and config 4 -----------------------------------------
        flush = torch.empty(2 * 126 * 2 ** 20 // 4, device=dev)
        pre = []
        for B, T, n in ((4, 8192, 3), (1, 65536, 2)):
            g = torch.Generator(device=dev).manual_seed(3)
            x3 = torch.randn(B, T, 3, H, D, device=dev, generator=g).to(torch.bfloat16)
            q, k, v = (x3[:, :, i].transpose(1, 2) for i in range(3))
            lg = F.logsigmoid(torch.randn(B, H, T, device=dev, generator=g) + 2.0)
            mix = torch.sigmoid(torch.randn(B, H, T, device=dev, generator=g)).to(torch.bfloat16)
            gs = torch.ones(1, H, 1, D, device=dev)
            y_ref, s_ref = ref_gla(q, k, v, lg, R, 64, mix_g=mix, gla_scale=gs)
            y_our = torch.empty_like(y_ref)
            s_our = torch.empty(B, H, J, D, device=dev)
            gla_forward(q, k, v, lg, R, mix_g=mix, gla_scale=gs, y=y_our, state_out=s_our)
            torch.cuda.synchronize()
            gla_diff = (y_ref.float() - y_our.float()).abs().max().item()
            state_diff = (s_ref[:, :, :J, :D] - s_our).abs().max().item()
            ref_attn(q, k, v, R, 2.0, mix, out=y_ref)
            exact_attention_triton(q, k, v, R, 2.0, mix, out=y_our)
            torch.cuda.synchronize()
            attn_diff = (y_ref.float() - y_our.float()).abs().max().item()
            t_gla = _event_ms(lambda: ref_gla(q, k, v, lg, R, 64, mix_g=mix, gla_scale=gs, out=y_ref), n, flush)
            t_attn = _event_ms(lambda: ref_attn(q, k, v, R, 2.0, mix, out=y_ref), n, flush)
            flops = B * H * (R + D) * T * T
            pre.append({"workload": f"prefill-B{B}-T{T}", "ms_by_kernel": {"gla": round(t_gla, 4),
                                                                            "outlier": round(t_attn, 4)},
                        "outlier_tflops": round(flops / (t_attn / 1e3) / 1e12, 1),
                        "maxabs_vs_ours": {"gla_y": gla_diff, "gla_state": state_diff, "y_after_attention": attn_diff}})
            del x3, y_ref, y_our
        out["prefill"] = pre
        # ---- the layer: forward at config 2, forward_step at config 1 (same weights as ours) -----
        torch.manual_seed(0)
        rcfg = RefConfig(d_model=1024, num_heads=H, num_layers=1, r=R, chunk_size=64)
        ref_layer = RefLayer(rcfg).to(dev).eval()
        with torch.no_grad():
            for name, prm in ref_layer.named_parameters():
                if "gate_proj.weight" in name or "mix_proj.weight" in name:
                    prm.normal_(0, 0.02)
        our_layer = HybridOutlierFactorizedAttention(ModelConfig(d_model=1024, num_heads=H, num_layers=1, r=R,
                                                                 chunk_size=64)).to(dev).eval()
        our_layer.load_state_dict(ref_layer.state_dict(), strict=True)
        x = torch.randn(4, 8192, 1024, device=dev, generator=torch.Generator(device=dev).manual_seed(8)) * 0.5
        lay = {}
        with torch.no_grad():
            # float32 (both libraries' float32 kernels).  The reference's inference layer uses
            # RMSNorm eps 1e-5 in its hybrid prefill, this layer float32 epsilon by default (the
            # reference's training layer and decode kernel): compared both ways
            xs32 = x[:1, :2048]
            y32 = ref_layer(xs32)
            lay["forward_fp32_B1_T2048_maxabs_vs_ours_default_eps"] = (y32 - our_layer(xs32)).abs().max().item()
            our_layer.hybrid_prefill_eps = 1e-5
            lay["forward_fp32_B1_T2048_maxabs_vs_ours_eps_1e-5"] = (y32 - our_layer(xs32)).abs().max().item()
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            yr = ref_layer(x)
            yo = our_layer(x)
            torch.cuda.synchronize()
            # bf16: the two differ in where they round (the reference divides the bf16
            # projection by d_h^(1/4), this library folds it into the weights; bf16 vs
            # float32 gate arithmetic), so the difference is compared with the output's size
            lay["forward_config2_maxabs_vs_ours_eps_1e-5"] = (yr.float() - yo.float()).abs().max().item()
            lay["forward_config2_max_abs_output"] = yr.float().abs().max().item()
            lay["forward_config2_ms"] = round(_event_ms(lambda: ref_layer(x), 3, flush), 4)
            lay["forward_config2_ms_ours"] = round(_event_ms(lambda: our_layer(x), 3, flush), 4)
        del x, yr, yo
        ref_bf = ref_layer.to(torch.bfloat16)
        for B in (1, 4):
            g = torch.Generator(device=dev).manual_seed(9)
            xs = torch.randn(B, 1, 1024, device=dev, generator=g).to(torch.bfloat16)
            caches = [((torch.randn(B, H, L, R, device=dev, generator=g) * KEY_STD).to(torch.bfloat16),
                       (torch.randn(B, H, L, D, device=dev, generator=g) * VAL_STD).to(torch.bfloat16))
                      for _ in range(4)]
            st = (torch.randn(B, H, J, D, device=dev, generator=g) * 0.1, torch.empty(B, H, J, D, device=dev))

            def launch(B=B, xs=xs, caches=caches, st=st):
                for i in range(64):
                    ref_bf.forward_step(xs, caches[i % 4], st, cache_seq_len=L - 1)

            with torch.no_grad():
                us = _decode_graph_time(launch, 64, 5, torch.cuda.Stream(dev))
            lay[f"forward_step_B{B}_us"] = round(us, 3)
        out["layer"] = lay
    except Exception as e:  # noqa: BLE001
        out["error"] = f"{type(e).__name__}: {e}"
    finally:
        if REF_DIR in sys.path:
            sys.path.remove(REF_DIR)
    return out


# ----------------------------------------------------------------------------- CPU arm
def cpu_baseline(B: int, seconds: float):
    """The reference's CPU computation of one decode step (oracle port of the
    training layer's decode core) on config-1 tensors, float32, all threads."""
    from oracle.hofa_oracle import FP32_EPS, decode_core
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    inp = make_step_inputs(B, "cpu", seed=1000, dtype=torch.float32)
    g = torch.Generator().manual_seed(5)
    ck = torch.randn(B, H, L, R, generator=g) * KEY_STD
    cv = torch.randn(B, H, L, D, generator=g) * VAL_STD
    st = torch.randn(B, H, J, D, generator=g) * 0.1
    step = lambda s: decode_core(inp["q"], inp["k"], inp["v"], ck, cv, s, inp["log_gamma"], inp["mix"].float(),
                                 inp["norm_w"], R, L, 2.0, eps=FP32_EPS, dtype=torch.float32)
    for _ in range(3):
        step(st)
    n, t0 = 0, time.perf_counter()
    while True:
        _, st = step(st)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    value = B * n / el
    return {"value": round(value, 2), "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} decode steps of config 1 (B={B}, L={L}) in float32, {el:.1f} s",
            "ms_per_step": round(1e3 * el / n, 3)}


def cpu_reference_layer(B: int, seconds: float):
    """The reference's own CPU PyTorch path for one decode step of the layer:
    ``HybridOutlierFactorizedAttentionTrain.forward_step``
    (src/HybridOutlierFactorizedAttentionTrain.py:298-438), imported
    unmodified from baseline/_ref, at config 1 (d_model 1024, H=16, r=16,
    B sequences with 4095 cached rows, so every step attends 4096), float32
    and bfloat16, all host threads; projections, gates, RoPE, the cache
    concatenation, the attention core and out_proj per step -- the work of
    this library's ``layer_step`` figure."""
    if not os.path.isdir(os.path.join(REF_DIR, "src")):
        return {"unavailable": "baseline/_ref is not installed"}
    sys.path.insert(0, REF_DIR)
    try:
        from src.config import ModelConfig as RefConfig
        from src.HybridOutlierFactorizedAttentionTrain import HybridOutlierFactorizedAttention as RefTrain
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import of the reference failed: {e!r}"}
    finally:
        if REF_DIR in sys.path:
            sys.path.remove(REF_DIR)
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    out = {"path": "HybridOutlierFactorizedAttentionTrain.forward_step, unmodified (baseline/_ref), CPU",
           "cores": torch.get_num_threads(), "workload": f"config1-layer-forward_step-B{B}-L{L}"}
    for dt in (torch.float32, torch.bfloat16):
        torch.manual_seed(0)
        layer = RefTrain(RefConfig(d_model=1024, num_heads=H, num_layers=1, r=R, chunk_size=64)).eval().to(dt)
        g = torch.Generator().manual_seed(6)
        x = torch.randn(B, 1, 1024, generator=g).to(dt)
        cache = ((torch.randn(B, H, L - 1, R, generator=g) * KEY_STD).to(dt),
                 (torch.randn(B, H, L - 1, D, generator=g) * VAL_STD).to(dt))
        state = torch.randn(B, H, D, D, generator=g) * 0.1
        state[:, :, J:] = 0
        with torch.no_grad():
            for _ in range(2):
                layer.forward_step(x, cache, state)
            n, t0 = 0, time.perf_counter()
            while True:
                layer.forward_step(x, cache, state)
                n += 1
                el = time.perf_counter() - t0
                if el >= seconds and n >= 3:
                    break
        out[str(dt).replace("torch.", "")] = {"ms_per_step": round(1e3 * el / n, 3), "tokens_per_s": round(B * n / el, 2),
                                               "steps": n}
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = cpu_baseline(args.batch, args.cpu_seconds)
    out = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": f"config1-decode-B{args.batch}-L{L}", "d_model": 1024, "heads": H, "d_head": D,
                      "r": R, "cache_len": L, "batch_per_gpu": args.batch,
                      "parallelism": "host CPU (reference PyTorch CPU path, oracle port)"},
           "cpu_baseline": {"value": cb["value"], "unit": "tokens/s", "cores": cb["cores"], "kind": "port",
                            "sample": cb["sample"]},
           "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--split-k", type=int, default=0)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config3", action="store_true", help="skip the 350M-shaped LM decode (config 3)")
    ap.add_argument("--no-triton-reference", action="store_true",
                    help="skip timing the reference's own Triton kernels (baseline/_ref)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-2 prefill measurement")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the config-4 (B=1, T=65536) prefill and long-cache decode measurement")
    ap.add_argument("--profile-config3", action="store_true",
                    help="only one graph replay of the 350M LM decode at --batch (for ncu captures)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="only the config-2 prefill kernels (for ncu captures); prints no bench line")
    ap.add_argument("--profile", action="store_true",
                    help="only warm-up + timed decode launches (for ncu captures); prints no bench line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.profile_config3:
        # small, self-contained command for ncu: one graph replay (two decode steps) of the 350M LM at B=1
        from outlierneuronattention_b200.lm import DecodeEngine, HofaLM, LMConfig
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        torch.manual_seed(0)
        model = HofaLM(LMConfig()).to(device=dev, dtype=torch.bfloat16).eval()
        idx = torch.randint(0, 32000, (args.batch, 16384), generator=torch.Generator().manual_seed(1)).to(dev)
        logits0, caches, states = model.prefill(idx, 16384 + 8, batch_chunk=8)
        eng = DecodeEngine(model, caches, states, logits0, 16384)
        eng.capture(4)
        eng.generate(2)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode")
        eng.generate(2)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"profile_config3": True, "batch": args.batch}))
    elif args.profile_prefill:
        # small, self-contained command for ncu: one warm-up and one timed prefill
        torch.cuda.set_device(0)
        print(json.dumps(measure_prefill(torch.device("cuda", 0), steps=1, warmup=1)))
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
