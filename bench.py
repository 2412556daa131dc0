"""Benchmark of the acefa attention engine on BASELINE config 2.

Workload (one "step"): the decode attention of a Qwen3-4B layer stack -- 36
ggml_flash_attn_ext ops, one per layer, each over that layer's own F16 KV cache
of 16 sets (8 requests x CFG cond/uncond), Hq=32 / Hkv=8, D=128, KV length
8192.  Inputs are seeded N(0,1) synthetic tensors resident in HBM; every layer's
KV (537 MB) is larger than L2, so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torchrun, one process per GPU; requests are sharded with no
collective on the data path (each rank owns a full 8-request batch: weak
scaling).  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "acestep.cpp_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

# ---- BASELINE config 2 (the metric's headline configuration) -------------
LAYERS, HQ, HKV, D = 36, 32, 8, 128
SETS, KV_LEN = 16, 8192
SEED = 42 + 1000 * 2
L2_BYTES = 126 * 1024 * 1024  # B200 L2: timed inputs exceed twice this or are flushed


def algo_bytes_per_op(sets=SETS, kv_len=KV_LEN, kv_bytes_per_row=2 * D, hq=HQ, hkv=HKV, d=D, mask=True):
    """Algorithmic HBM bytes of one decode op: K+V rows read once, Q read,
    O written (f32), mask read once per set."""
    kv = sets * hkv * kv_len * kv_bytes_per_row * 2
    qo = sets * hq * d * 4 * 2
    m = sets * kv_len * 2 if mask else 0
    return kv + qo + m


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def read_traffic(kernel_key):
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    try:
        with open(p) as f:
            return json.load(f).get(kernel_key, {}).get("dram_bytes_per_launch")
    except Exception:
        return None


class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU sampled DURING the
    timed region: an NVML polling thread (every 2 ms; reads only), so even a
    timed region of a few tens of milliseconds gets samples.  Falls back to
    `nvidia-smi -lms 200` when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.rows = []
        self.nvml = None
        self.handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(index).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nvml = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nvml = None
        self.tmpdir = tempfile.mkdtemp(prefix="acefa_clocks_")
        self.path = os.path.join(self.tmpdir, f"clocks_rank{index}.csv")

    def _poll(self):
        import time

        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop:
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                bits = int(get_reasons(self.handle))
                self.rows.append((mhz, self.max_mhz, [n for n, b in self.REASONS.items() if bits & b]))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nvml is not None:
            import threading

            self.stop = False
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.nvml is not None:
            self.stop = True
            self.thread.join(timeout=5)
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        rows = list(self.rows)
        if self.nvml is None:
            if self.proc is None or not os.path.exists(self.path):
                return None
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]),
                                 [names[i] for i, v in enumerate(parts[5:9]) if v.lower() == "active"]))
                except ValueError:
                    continue
        if not rows:
            return None
        reasons = sorted({n for _, _, r in rows for n in r})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# -------------------------------------------------------------------------
def cpu_baseline(budget_s=12.0, threads=None, half=False):
    """The reference operator's CPU arithmetic (oracle, ggml-cpu mode) on a
    bounded sample of the same workload: whole layers of config 2."""
    import numpy as np

    import oracle

    threads = threads or os.cpu_count()
    rng = np.random.default_rng(SEED)
    q = rng.standard_normal((SETS, HQ, 1, D), dtype=np.float32)
    k = rng.standard_normal((SETS, HKV, KV_LEN, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((SETS, HKV, KV_LEN, D), dtype=np.float32).astype(np.float16)
    m = np.zeros((SETS, 1, 1, KV_LEN), np.float16)
    oracle.flash_attn_ext(q[:1], k[:1], v[:1], m[:1], scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.flash_attn_ext(q, k, v, m, scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=threads)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s or n >= 5000:
            break
    gbs = n * algo_bytes_per_op() / dt / 1e9
    hw2 = None
    if threads > 1 and not half:
        hw2 = cpu_baseline(budget_s=budget_s / 2, threads=max(1, threads // 2), half=True)
        hw2 = {"value": hw2["value"], "cores": hw2["cores"]}
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "hw2": hw2,
            "sample": f"{n} layer(s) of the config-2 decode op (16 sets x 8192 keys, F16 KV) in {dt:.1f} s; "
                      f"oracle/fa_oracle.c ggml-cpu arithmetic, OpenMP"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    import oracle

    threads = os.cpu_count()
    rng = np.random.default_rng(SEED)
    q = rng.standard_normal((SETS, HQ, 1, D), dtype=np.float32)
    k = rng.standard_normal((SETS, HKV, KV_LEN, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((SETS, HKV, KV_LEN, D), dtype=np.float32).astype(np.float16)
    m = np.zeros((SETS, 1, 1, KV_LEN), np.float16)

    def step():  # one bounded sample: one layer of the stack
        oracle.flash_attn_ext(q, k, v, m, scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    gbs = args.steps * algo_bytes_per_op() / dt / 1e9
    line = {
        "impl": "reference", "metric": "decode_attention_hbm_gbs", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,1), seed 2042",
        "config": config_dict(args, note="one step = one layer of the stack on the host CPU"),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "one layer (16 sets x 8192 keys) per step; the reference's ggml "
                                   "kernels are absent from its tree, so the CPU restatement "
                                   "(oracle/fa_oracle.c, ggml-cpu arithmetic) stands in"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


def config_dict(args, note=None):
    layers = getattr(args, "layers", LAYERS)
    kv = getattr(args, "kv", "f16")
    c = {"workload": f"qwen3-4b decode attention stack (BASELINE config 2): {layers} layers x ggml_flash_attn_ext, "
                     f"8 requests x CFG = 16 KV sets, Hq 32 / Hkv 8, D 128, KV 8192, {kv.upper()} KV, "
                     "mask [8192,1,1,16]",
         "layers": layers, "kv_sets_per_gpu": SETS, "kv_len": KV_LEN, "head_dim": D, "q_heads": HQ,
         "kv_heads": HKV, "kv_type": kv, "l2": "inputs larger than L2 (537 MB of KV per op); no flush",
         "parallelism": f"requests sharded one batch per GPU x{args.gpus}, no collective"}
    if note:
        c["note"] = note
    return c


# -------------------------------------------------------------------------
def build_stack(device, kv="f16", layers=LAYERS, sets=SETS, kv_len=KV_LEN, seed=SEED, valid=None):
    """`layers` distinct decode ops over caches of kv_len rows; valid < kv_len
    masks rows valid.. to -inf (the reference's padded decode window)."""
    import torch

    import acefa

    g = torch.Generator(device=device).manual_seed(seed)
    ops, hosts = [], []
    mask = torch.zeros(sets, 1, 1, kv_len, device=device, dtype=torch.float16)
    if valid is not None:
        mask[..., valid:] = float("-inf")
    ws = None
    for _ in range(layers):
        q = torch.randn(sets, HQ, 1, D, device=device, generator=g)
        kf = torch.randn(sets, HKV, kv_len, D, device=device, generator=g, dtype=torch.float16)
        vf = torch.randn(sets, HKV, kv_len, D, device=device, generator=g, dtype=torch.float16)
        if kv == "q8_0":
            k, v, kt = acefa.quantize_q8_0(kf), acefa.quantize_q8_0(vf), acefa.GGML_Q8_0
            del kf, vf
        else:
            k, v, kt = kf, vf, None
        op = acefa.Op(q, k, v, mask=mask, kv_type=kt, scale=D ** -0.5)
        if ws is None or ws.numel() < op.workspace.numel():
            ws = op.workspace
        ops.append(op)
    for op in ops:  # one pooled workspace, like ggml-cuda's pool (ops run stream-ordered)
        op.workspace = ws
    return ops, mask


def time_graph(ops, steps, warmup, stream):
    import torch

    for _ in range(2):
        for op in ops:
            op(stream=stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for op in ops:
            op(stream=stream)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    return graph


def run_ours(args):
    import torch
    import torch.distributed as dist

    import acefa

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    stream = torch.cuda.Stream(device=device)
    row_bytes = D // 32 * 34 if args.kv == "q8_0" else 2 * D
    per_op = algo_bytes_per_op(kv_bytes_per_row=row_bytes)
    with torch.cuda.stream(stream):
        ops, mask = build_stack(device, kv=args.kv, layers=args.layers, seed=SEED + 7919 * rank)
        launches_per_op = 0
        ops[0](stream=stream)
        launches_per_op = acefa.last_launch_count()
        graph = time_graph(ops, args.steps, max(args.warmup, 3), stream)

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()  # replays on the current stream
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    step_bytes = per_op * args.layers
    value = world * step_bytes * args.steps / (ms_max / 1e3) / 1e9
    assert acefa.device_error(stream) == 0

    # ---- end to end through the C ABI with host buffers ----------------------
    q_host = [torch.empty_like(op.q, device="cpu").pin_memory() for op in ops]
    for qh, op in zip(q_host, ops):
        qh.copy_(op.q)
    m_host = torch.empty_like(mask, device="cpu").pin_memory()
    m_host.copy_(mask)
    o_host = [torch.empty_like(op.out, device="cpu").pin_memory() for op in ops]
    e2e_steps = max(2, min(args.steps, 10))

    # Copies run on their own streams, as a serving loop would issue them: layer
    # l's Q goes up while earlier layers compute, its output comes down while
    # later layers compute.  Events keep every buffer's reuse ordered across
    # steps (a Q buffer is refilled only after its op of the previous step ran,
    # an output is overwritten only after its previous copy-out finished).
    up, down = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    L_ops = len(ops)
    ev_in = [torch.cuda.Event() for _ in range(L_ops)]     # Q_l on the device
    ev_ran = [torch.cuda.Event() for _ in range(L_ops)]    # op l finished
    ev_out = [torch.cuda.Event() for _ in range(L_ops)]    # out_l on the host
    ev_mask = torch.cuda.Event()
    started = [False]

    def e2e_step():
        with torch.cuda.stream(up):
            if started[0]:
                up.wait_event(ev_ran[L_ops - 1])  # every op of the last step has read the mask
            mask.copy_(m_host, non_blocking=True)
            ev_mask.record(up)
            for l, (qh, op) in enumerate(zip(q_host, ops)):
                if started[0]:
                    up.wait_event(ev_ran[l])
                op.q.copy_(qh, non_blocking=True)
                ev_in[l].record(up)
        stream.wait_event(ev_mask)
        for l, op in enumerate(ops):
            stream.wait_event(ev_in[l])
            if started[0]:
                stream.wait_event(ev_out[l])
            op(stream=stream)
            ev_ran[l].record(stream)
        with torch.cuda.stream(down):
            for l, (oh, op) in enumerate(zip(o_host, ops)):
                down.wait_event(ev_ran[l])
                oh.copy_(op.out, non_blocking=True)
                ev_out[l].record(down)
        started[0] = True

    with torch.cuda.stream(stream):
        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        up.wait_event(e0)
        for _ in range(e2e_steps):
            e2e_step()
        stream.wait_event(ev_out[L_ops - 1])  # the last copy-out is inside the timed region
        e1.record(stream)
        torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_gbs = world * step_bytes * e2e_steps / (float(te.item()) / 1e3) / 1e9
    h2d = mask.numel() * mask.element_size() + sum(op.q.numel() * 4 for op in ops)
    d2h = sum(op.out.numel() * 4 for op in ops)

    out = None
    if rank == 0:
        peak, peak_kind = read_peaks()
        per_launch_s = (ms_step / 1e3) / args.layers
        achieved = per_op / per_launch_s / 1e9
        out = {
            "metric": "decode_attention_hbm_gbs", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.kv,
            "data": "synthetic N(0,1) K/V/Q, seeded (2042 + 7919*rank); random values, zero mask",
            "config": config_dict(args),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": read_traffic(f"fa_decode_kernel_{args.kv}_d128"),
                         "peak_source": f"{peak_kind} hbm_gbs", "kernel": f"fa_decode_kernel<{args.kv},128>",
                         "algo_bytes_per_launch": per_op},
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "how": "pinned H2D of mask + 36 Q, 36 C-ABI calls, D2H of 36 outputs; copies on their own streams overlap the ops; CUDA events"},
            "gpu_launches": int(launches_per_op * args.layers * args.steps),
            "clocks": clk.summary(),
        }
    # free the F16 stack before optional extras
    del graph, ops
    torch.cuda.empty_cache()

    if rank == 0 and not args.no_extras:
        out["extras"] = extras(device, stream, args)
        out["extras"]["dense"] = dense_extras(device, stream, cpu=not args.no_cpu_baseline)
        out["extras"]["config2_sweep"] = decode_sweep(device, stream)
    if world > 1 and not args.no_extras:
        sharded = sharded_dit(device, stream, world, rank)  # collective: every rank
        if rank == 0:
            out["extras"]["dit6000_heads_sharded"] = sharded
    if not args.no_extras and not args.no_config5:
        c5 = config5(device, stream, world, rank, gen=args.c5_gen)  # collective at N > 1: every rank
        if rank == 0:
            out["extras"]["config5"] = c5
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
            if "config5" in out.get("extras", {}):
                out["extras"]["config5"]["cpu_baseline"] = config5_cpu_baseline()
        emit(out)
    return 0


def extras(device, stream, args):
    """Secondary figures on rank 0: Q8_0 KV stack and the config-1 single op."""
    import torch

    res = {}
    peak, _ = read_peaks()
    with torch.cuda.stream(stream):
        ops, _ = build_stack(device, kv="q8_0", seed=SEED + 1)
        graph = time_graph(ops, 5, 3, stream)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(5):
            graph.replay()
        s1.record(stream)
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1) / 5
        qb = algo_bytes_per_op(kv_bytes_per_row=D // 32 * 34) * LAYERS
        res["q8_0_stack"] = {"gbs": round(qb / (ms / 1e3) / 1e9, 1), "ms_per_step": round(ms, 4),
                             "frac_of_hbm_peak": round(qb / (ms / 1e3) / 1e9 / peak, 4)}
        del graph, ops
        torch.cuda.empty_cache()
        # config 1: one Qwen3-0.6B decode op (8.4 MB), many back-to-back in a graph
        import acefa

        reps = 64
        b1 = 8_409_088
        for key, rule in (("config1_single_op", False), ("config1_single_op_rule", True)):
            g = torch.Generator(device=device).manual_seed(42 + 1000)
            ops = []
            for _ in range(reps):
                q = torch.randn(1, 16, 1, D, device=device, generator=g)
                k = torch.randn(1, 8, 2048, D, device=device, generator=g, dtype=torch.float16)
                v = torch.randn(1, 8, 2048, D, device=device, generator=g, dtype=torch.float16)
                if rule:  # the same visibility (keys 0 .. 2047) by rule: no mask read
                    ops.append(acefa.Op(q, k, v, mask_gen=acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[2047]),
                                        scale=D ** -0.5))
                else:
                    m = torch.zeros(1, 1, 1, 2048, device=device, dtype=torch.float16)
                    ops.append(acefa.Op(q, k, v, mask=m, scale=D ** -0.5))
            graph = time_graph(ops, 10, 3, stream)
            s0.record(stream)
            for _ in range(10):
                graph.replay()
            s1.record(stream)
            torch.cuda.synchronize()
            us = s0.elapsed_time(s1) * 1e3 / (10 * reps)
            gbs = b1 / (us / 1e6) / 1e9
            res[key] = {"us_per_op": round(us, 2), "gbs": round(gbs, 1),
                        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                     "frac": round(gbs / peak, 4),
                                     "traffic": read_traffic("fa_decode_kernel_f16_config1"),
                                     "algo_bytes_per_launch": b1},
                        "note": "64 distinct ops back to back in one CUDA graph (8.4 MB each)" +
                                ("; mask by rule" if rule else "")}
            if not rule:
                res[key]["e2e"] = config1_e2e(ops, stream, b1)
            del graph, ops
        if not getattr(args, "no_cpu_baseline", False):
            res["config1_single_op"]["cpu_baseline"] = config1_cpu_baseline()
        res["config1_append"] = append_step(device, stream)
        res["dit6000_prologue"] = dit_prologue(device, stream)
        res["cfg_logit_combine"] = cfg_combine_step(device, stream)
    return res


def config1_e2e(ops, stream, nbytes, iters=5):
    """Config 1 through the C ABI with host buffers: per op the pinned H2D of
    Q and the mask, the call, the D2H of the output (64 ops per round, copies
    on their own streams as a serving loop issues them)."""
    import torch

    up, down = torch.cuda.Stream(device=stream.device), torch.cuda.Stream(device=stream.device)
    qh = [torch.empty_like(op.q, device="cpu").pin_memory() for op in ops]
    mh = [torch.empty_like(op.mask, device="cpu").pin_memory() for op in ops]
    oh = [torch.empty_like(op.out, device="cpu").pin_memory() for op in ops]
    ev_in = [torch.cuda.Event() for _ in ops]
    ev_ran = [torch.cuda.Event() for _ in ops]

    def rnd():
        with torch.cuda.stream(up):
            for i, op in enumerate(ops):
                op.q.copy_(qh[i], non_blocking=True)
                op.mask.copy_(mh[i], non_blocking=True)
                ev_in[i].record(up)
        for i, op in enumerate(ops):
            stream.wait_event(ev_in[i])
            op(stream=stream)
            ev_ran[i].record(stream)
        with torch.cuda.stream(down):
            for i, op in enumerate(ops):
                down.wait_event(ev_ran[i])
                oh[i].copy_(op.out, non_blocking=True)

    rnd()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    for _ in range(iters):
        rnd()
        torch.cuda.synchronize()  # rounds do not overlap: every buffer is reused
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (iters * len(ops))
    h2d = ops[0].q.numel() * 4 + ops[0].mask.numel() * 2
    return {"us_per_op": round(us, 2), "gbs": round(nbytes / (us / 1e6) / 1e9, 1), "h2d_bytes_per_op": int(h2d),
            "d2h_bytes_per_op": int(ops[0].out.numel() * 4),
            "how": "pinned H2D of Q + mask, C-ABI call, D2H of the output per op; copies on their own streams"}


def config1_cpu_baseline(budget_s=2.0):
    """The config-1 op on the host cores (oracle, ggml-cpu arithmetic), at nproc
    and at the reference's default of hw/2 threads (src/backend.h:28-31)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(42 + 1000)
    q = rng.standard_normal((1, 16, 1, D), dtype=np.float32)
    k = rng.standard_normal((1, 8, 2048, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((1, 8, 2048, D), dtype=np.float32).astype(np.float16)
    m = np.zeros((1, 1, 1, 2048), np.float16)
    out = {}
    for label, th in (("nproc", os.cpu_count()), ("hw2", max(1, (os.cpu_count() or 2) // 2))):
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.flash_attn_ext(q, k, v, m, scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=th)
            n += 1
        dt = time.perf_counter() - t0
        out[label] = {"us_per_op": round(dt / n * 1e6, 1), "gbs": round(n * 8_409_088 / dt / 1e9, 2), "cores": th}
    return {"value": out["nproc"]["gbs"], "unit": "GB/s", "cores": out["nproc"]["cores"], "kind": "port",
            "us_per_op": out["nproc"]["us_per_op"], "hw2": out["hw2"],
            "sample": "the config-1 op repeated for ~2 s per thread count; oracle/fa_oracle.c ggml-cpu arithmetic"}


def append_step(device, stream, reps=64, kv_len=2048):
    """A config-1 decode step with its KV-cache append: the new K and V rows
    written by two separate row writes (standing in for ggml_set_rows) and then
    the attention, against acefa_flash_attn_ext_append doing both in one
    launch.  64 distinct layers back to back in one CUDA graph each."""
    import torch

    import acefa

    g = torch.Generator(device=device).manual_seed(42 + 1000 + 7)
    wq = 1.0 + 0.1 * torch.randn(D, device=device, generator=g)
    wk = 1.0 + 0.1 * torch.randn(D, device=device, generator=g)
    pos32 = torch.tensor([kv_len - 1], dtype=torch.int32, device=device)
    cos, sin = rope_table(pos32, device)
    sep, fused, sep_pro, fused_pro = [], [], [], []
    for _ in range(reps):
        q = torch.randn(1, 16, 1, D, device=device, generator=g)
        k = torch.randn(1, 8, kv_len, D, device=device, generator=g, dtype=torch.float16)
        v = torch.randn(1, 8, kv_len, D, device=device, generator=g, dtype=torch.float16)
        m = torch.zeros(1, 1, 1, kv_len, device=device, dtype=torch.float16)
        kn = torch.randn(1, 8, 1, D, device=device, generator=g)
        vn = torch.randn(1, 8, 1, D, device=device, generator=g)
        pos = torch.tensor([kv_len - 1], dtype=torch.int64, device=device)
        op = acefa.Op(q, k, v, mask=m, scale=D ** -0.5)
        sep.append((op, k, v, kn, vn, pos))
        fused.append(acefa.Op(q, k, v, mask=m, scale=D ** -0.5, k_new=kn, v_new=vn, pos=pos))
        # with the QK-norm + RoPE prologue: torch ops then the operator, or all in one call
        qr = torch.empty_like(q)
        sep_pro.append((acefa.Op(qr, k, v, mask=m, scale=D ** -0.5), q, qr, k, v, kn, vn, pos))
        fused_pro.append(acefa.Op(q, k, v, mask=m, scale=D ** -0.5, k_new=kn, v_new=vn, pos=pos,
                                  q_prologue=acefa.RopeNorm(wq, 1e-6, 1.0e6, pos32),
                                  k_prologue=acefa.RopeNorm(wk, 1e-6, 1.0e6, pos32)))

    def run_sep():
        for op, k, v, kn, vn, pos in sep:
            k.index_copy_(2, pos, kn.half())
            v.index_copy_(2, pos, vn.half())
            op(stream=torch.cuda.current_stream())

    def run_fused():
        for op in fused:
            op(stream=torch.cuda.current_stream())

    def run_sep_pro():
        for op, q, qr, k, v, kn, vn, pos in sep_pro:
            qr.copy_(torch_rope_norm(q, wq, cos, sin))
            k.index_copy_(2, pos, torch_rope_norm(kn, wk, cos, sin).half())
            v.index_copy_(2, pos, vn.half())
            op(stream=torch.cuda.current_stream())

    def run_fused_pro():
        for op in fused_pro:
            op(stream=torch.cuda.current_stream())

    out = {}
    for name, fn in (("separate_us_per_step", run_sep), ("fused_us_per_step", run_fused),
                     ("separate_with_prologue_us_per_step", run_sep_pro),
                     ("fused_with_prologue_us_per_step", run_fused_pro)):
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                fn()
            for _ in range(3):
                graph.replay()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(10):
                graph.replay()
            s1.record(stream)
            torch.cuda.synchronize()
        out[name] = round(s0.elapsed_time(s1) * 1e3 / (10 * reps), 2)
        del graph
    out["note"] = ("config-1 shape, new row at the last position; separate = two row writes (torch index_copy, "
                   "standing in for ggml_set_rows) + acefa_flash_attn_ext; with_prologue adds QK-norm + RoPE of "
                   "Q and the new K row (torch ops standing in for ggml's rms_norm / mul / rope nodes, vs fused "
                   "into the same single launch)")
    return out


def cfg_combine_step(device, stream, n=8, reps=64, iters=10):
    """The CFG combine + compaction of one batched decode step (8 requests,
    partial LM head: out_V = 65559, EOS + 65535 codes; src/pipeline-lm.cpp:
    471-492).  Device: acefa_cfg_logit_combine over 64 distinct logit buffers
    (269 MB > L2) in one CUDA graph.  Host paths, wall clock per step: the
    reference's (D2H of all 2n rows into pinned memory, then its loop, here the
    oracle's C restatement on one core) against ours (the launch plus the D2H
    of the compact rows)."""
    import time

    import numpy as np
    import torch

    import acefa

    out_v, eos, off, cnt = 65559, 0, 24, 65535
    g = torch.Generator(device=device).manual_seed(SEED + 77)
    bufs = [torch.randn(2 * n, out_v, device=device, generator=g) * 10 for _ in range(reps)]
    outs = [torch.empty(n, cnt + 1, device=device) for _ in range(reps)]
    peak, _ = read_peaks()
    with torch.cuda.stream(stream):
        def run():
            for b, o in zip(bufs, outs):
                acefa.cfg_logit_combine(b[:n], b[n:], eos, off, cnt, 2.0, out=o, stream=stream)
        run()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        for _ in range(3):
            graph.replay()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(iters):
            graph.replay()
        s1.record(stream)
        torch.cuda.synchronize()
    us = s0.elapsed_time(s1) * 1e3 / (iters * reps)
    algo = n * (cnt + 1) * 4 * 3  # cond + uncond columns read, compact written
    gbs = algo / (us / 1e6) / 1e9
    del graph
    # host-side step, as the sampler sees it
    import oracle as ora

    full_h = torch.empty(2 * n, out_v, pin_memory=True)
    comp_h = torch.empty(n, cnt + 1, pin_memory=True)
    b, o = bufs[0], outs[0]

    def ref_step():
        full_h.copy_(b, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        fh = full_h.numpy()
        return ora.cfg_logit_combine(fh[:n], fh[n:], eos, off, cnt, 2.0)

    def our_step():
        acefa.cfg_logit_combine(b[:n], b[n:], eos, off, cnt, 2.0, out=o)
        comp_h.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return comp_h.numpy()

    res = {}
    for name, fn in (("reference_host_us_per_step", ref_step), ("device_combine_us_per_step", our_step)):
        for _ in range(3):
            fn()
        t0 = time.perf_counter()
        for _ in range(20):
            fn()
        res[name] = round((time.perf_counter() - t0) / 20 * 1e6, 1)
    assert np.array_equal(ref_step(), our_step().copy())
    del bufs, outs
    return {"us_per_launch": round(us, 3), "gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "algo_bytes_per_launch": algo,
                         "traffic": read_traffic("cfg_logit_combine_kernel")},
            "d2h_bytes_per_step": {"reference": 2 * n * out_v * 4, "device_combine": n * (cnt + 1) * 4},
            **res,
            "note": "64 distinct 4.2 MB logit buffers back to back in one CUDA graph; host steps by wall "
                    "clock incl. the D2H (pinned) and synchronisation; results bit-identical"}


def rope_table(pos, device, theta=1.0e6):
    """cos / sin (rows, D/2) of RoPE NEOX for int positions (torch reference path)."""
    import torch

    inv = theta ** (-torch.arange(0, D, 2, device=device, dtype=torch.float32) / D)
    a = pos.float()[:, None] * inv[None, :]
    return a.cos(), a.sin()


def torch_rope_norm(x, w, cos, sin, eps=1e-6):
    """RMSNorm * w then RoPE NEOX over the last axis, as separate torch kernels
    (the stand-in for the reference's rms_norm, mul and rope graph nodes).
    cos / sin broadcast against x's rows (..., rows, D/2)."""
    import torch

    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
    y1, y2 = y[..., : D // 2], y[..., D // 2:]
    return torch.cat([y1 * cos - y2 * sin, y1 * sin + y2 * cos], dim=-1)


def dit_prologue(device, stream, N=2, H=16, S=6000, iters=10):
    """A DiT self-attention layer's prologue + attention (config-4 shape):
    separate = torch rms_norm / mul / rope / cast / permute kernels (standing in
    for the reference's graph nodes) then acefa_flash_attn_ext, against
    acefa_kv_prologue + the operator with the Q prologue fused."""
    import torch

    import acefa

    g = torch.Generator(device=device).manual_seed(42 + 2000)
    # projections as the DiT graph leaves them: [D, H, S, N] f32 = torch (N, S, H, D)
    q_raw = torch.randn(N, S, H, D, device=device, generator=g)
    k_raw = torch.randn(N, S, H, D, device=device, generator=g)
    v_raw = torch.randn(N, S, H, D, device=device, generator=g)
    wq = 1.0 + 0.1 * torch.randn(D, device=device, generator=g)
    wk = 1.0 + 0.1 * torch.randn(D, device=device, generator=g)
    pos = torch.arange(S, device=device, dtype=torch.int32).repeat(N)
    cos, sin = rope_table(torch.arange(S, device=device, dtype=torch.int32), device)
    cos, sin = cos[None, :, None, :], sin[None, :, None, :]  # against (N, S, H, D/2)
    qs = torch.empty(N, H, S, D, device=device)
    k16 = torch.empty(N, H, S, D, device=device, dtype=torch.float16)
    v16 = torch.empty_like(k16)
    op_sep = acefa.Op(qs, k16, v16, scale=D ** -0.5)
    op_fused = acefa.Op(q_raw.permute(0, 2, 1, 3), k16, v16, scale=D ** -0.5,
                        q_prologue=acefa.RopeNorm(wq, 1e-6, 1.0e6, pos))
    k_pro = acefa.RopeNorm(wk, 1e-6, 1.0e6, pos)

    def run_sep():
        qs.copy_(torch_rope_norm(q_raw, wq, cos, sin).permute(0, 2, 1, 3))
        k16.copy_(torch_rope_norm(k_raw, wk, cos, sin).permute(0, 2, 1, 3))
        v16.copy_(v_raw.permute(0, 2, 1, 3))
        op_sep(stream=torch.cuda.current_stream())

    def run_fused():
        st = torch.cuda.current_stream()
        acefa.kv_prologue(k_raw.permute(0, 2, 1, 3), k16, v_raw.permute(0, 2, 1, 3), v16, k_pro, stream=st)
        op_fused(stream=st)

    out = {}
    for name, fn in (("separate_ms", run_sep), ("fused_ms", run_fused)):
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                fn()
            for _ in range(3):
                graph.replay()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(iters):
                graph.replay()
            s1.record(stream)
            torch.cuda.synchronize()
        out[name] = round(s0.elapsed_time(s1) / iters, 4)
        del graph
    # the prologue pass alone: K and V read as f32, written as f16
    with torch.cuda.stream(stream):
        st = stream
        for _ in range(3):
            acefa.kv_prologue(k_raw.permute(0, 2, 1, 3), k16, v_raw.permute(0, 2, 1, 3), v16, k_pro, stream=st)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(iters):
            acefa.kv_prologue(k_raw.permute(0, 2, 1, 3), k16, v_raw.permute(0, 2, 1, 3), v16, k_pro, stream=st)
        s1.record(stream)
        torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / iters
    nbytes = 2 * N * S * H * D * (4 + 2)
    peak, _ = read_peaks()
    out["kv_prologue_ms"] = round(ms, 4)
    out["kv_prologue_gbs"] = round(nbytes / (ms / 1e3) / 1e9, 1)
    out["kv_prologue_frac_of_hbm_peak"] = round(nbytes / (ms / 1e3) / 1e9 / peak, 4)
    out["note"] = "N=2 x H=16 x S=6000, D=128; separate = torch kernels standing in for the reference's graph nodes"
    return out


def decode_sweep(device, stream, layers=LAYERS):
    """BASELINE config 2's sweep: KV length {512, 2048, 8192} x KV sets
    {2, 8, 16} (1, 4, 8 requests x CFG) x F16 / Q8_0, each a stack of `layers`
    distinct layers replayed in one CUDA graph (the (8192, 16) points are the
    headline and the q8_0_stack figures), plus the padded decode windows
    PAD(L + 1, 256) at 16 sets."""
    import torch

    peak, _ = read_peaks()
    res = {}
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for kv in ("f16", "q8_0"):
        row = 2 * D if kv == "f16" else D // 32 * 34
        for kv_len in (512, 2048, 8192):
            for sets in (2, 8, 16):
                if kv_len == 8192 and sets == 16:
                    continue
                # at least twice the L2 of distinct layers, so that no replay
                # finds its K/V in L2 (36 layers of the smallest points hold
                # less than the L2)
                per_op = algo_bytes_per_op(sets=sets, kv_len=kv_len, kv_bytes_per_row=row)
                nl = max(layers, -(-2 * L2_BYTES // per_op))
                with torch.cuda.stream(stream):
                    ops, _ = build_stack(device, kv=kv, layers=nl, sets=sets, kv_len=kv_len,
                                         seed=SEED + 17 * kv_len + sets)
                    graph = time_graph(ops, 5, 3, stream)
                    s0.record(stream)
                    for _ in range(5):
                        graph.replay()
                    s1.record(stream)
                    torch.cuda.synchronize()
                ms = s0.elapsed_time(s1) / 5
                b = per_op * nl
                gbs = b / (ms / 1e3) / 1e9
                res[f"L{kv_len}_N{sets}_{kv}"] = {"gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / peak, 4),
                                                  "us_per_op": round(ms * 1e3 / nl, 2), "layers": int(nl)}
                del graph, ops
                torch.cuda.empty_cache()
        # the padded window of a decode step (n_kv_pad = PAD(L + 1, 256), rows
        # past L masked): the dead tail tiles are skipped; bytes count the valid
        # K/V rows and the whole mask
        for kv_len in (2048, 8192):
            win = pad256(kv_len + 1)
            with torch.cuda.stream(stream):
                ops, _ = build_stack(device, kv=kv, layers=layers, sets=16, kv_len=win, valid=kv_len,
                                     seed=SEED + 19 * kv_len)
                graph = time_graph(ops, 5, 3, stream)
                s0.record(stream)
                for _ in range(5):
                    graph.replay()
                s1.record(stream)
                torch.cuda.synchronize()
            ms = s0.elapsed_time(s1) / 5
            b = (algo_bytes_per_op(sets=16, kv_len=kv_len, kv_bytes_per_row=row) + 16 * (win - kv_len) * 2) * layers
            gbs = b / (ms / 1e3) / 1e9
            res[f"L{kv_len}_pad{win}_N16_{kv}"] = {"gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / peak, 4),
                                                    "us_per_op": round(ms * 1e3 / layers, 2)}
            del graph, ops
            torch.cuda.empty_cache()
    return res


# -------------------------------------------------------------------------
# dense path (BASELINE configs 3 and 4): TFLOP/s over unmasked (q, k) pairs
DENSE_WORKLOADS = {
    # name: (B, Hq, Hkv, S_q, S_kv, mask kind, extra)
    "prefill1024": (2, 16, 8, 1024, 1024, "causal", None),
    "prefill4096": (2, 16, 8, 4096, 4096, "causal", None),
    "dit1500": (2, 16, 16, 1500, 1500, None, None),
    "dit6000": (2, 16, 16, 6000, 6000, None, None),
    "dit6000_window128": (2, 16, 16, 6000, 6000, "window", 128),
    "cross6000": (2, 16, 16, 6000, 512, "padding", 461),
    # the real DiT has 8 K/V heads (GQA-2) and S = T / patch_size: S = 1085 in
    # the reference's logs, 750 / 3000 for 30 s / 120 s of audio
    "dit1085_gqa8": (2, 16, 8, 1085, 1085, None, None),
    "dit750": (2, 16, 16, 750, 750, None, None),
    "dit3000": (2, 16, 16, 3000, 3000, None, None),
    "dit6000_gqa8": (2, 16, 8, 6000, 6000, None, None),
    # BF16 inputs (config 4 names "BF16/F16 inputs") and the config-5 prompt
    # prefill over a Q8_0 KV cache (one set: Q [128, 512, 32], K/V [128, 512, 8])
    "dit6000_bf16": (2, 16, 16, 6000, 6000, None, None, "bf16"),
    "prefill512_q8_0": (1, 32, 8, 512, 512, "causal", None, "q8_0"),
    # head dims 64 (tcgen05, N = 64 PV) and 256 (F16 / BF16 only, on the
    # split-KV kernel): operator shapes ggml accepts, not used by acestep.cpp
    "dit6000_d64": (2, 16, 16, 6000, 6000, None, None, "f16", 64),
    "dit1500_d256": (2, 16, 16, 1500, 1500, None, None, "f16", 256),
}
# workloads whose CPU baseline (oracle on sampled query rows) is timed too
DENSE_CPU_SAMPLED = ("prefill4096", "dit6000", "cross6000")


def dense_pairs(S_q, S_kv, kind, extra):
    if kind is None:
        return S_q * S_kv
    if kind == "causal":
        return S_q * (S_q + 1) // 2
    if kind == "padding":
        return S_q * extra
    if kind == "window":
        i = __import__("numpy").arange(S_q)
        return int((__import__("numpy").minimum(S_kv - 1, i + extra) - __import__("numpy").maximum(0, i - extra) + 1).sum())
    raise ValueError(kind)


def dense_bytes(name, rule=False):
    """Algorithmic HBM bytes of one dense op: Q read and O written in f32, K
    and V read once (F16/BF16 2 B per value, Q8_0 34 B per 32 values), the f16
    mask read once (none when the mask is given by rule)."""
    B, Hq, Hkv, S_q, S_kv, kind, extra = DENSE_WORKLOADS[name][:7]
    kv = DENSE_WORKLOADS[name][7] if len(DENSE_WORKLOADS[name]) > 7 else "f16"
    hd = DENSE_WORKLOADS[name][8] if len(DENSE_WORKLOADS[name]) > 8 else D
    kv_row = hd * 34 // 32 if kv == "q8_0" else hd * 2
    qo = 2 * B * Hq * S_q * hd * 4
    kvb = 2 * B * Hkv * S_kv * kv_row
    m = S_q * S_kv * 2 if (kind is not None and not rule) else 0
    return qo + kvb + m


def dense_bound(flops, nbytes, ms, tflops_peak, hbm_peak):
    """The op's roofline: its shortest possible time is the longer of the
    tensor time (FLOPs / tensor peak) and the HBM time (bytes / HBM peak);
    `bound` names the longer one and `frac_of_bound` = that time / measured."""
    t_tensor = flops / (tflops_peak * 1e12) * 1e3
    t_hbm = nbytes / (hbm_peak * 1e9) * 1e3
    bound = "tensor" if t_tensor >= t_hbm else "hbm"
    return {"bound": bound, "tensor_ms": round(t_tensor, 5), "hbm_ms": round(t_hbm, 5),
            "frac_of_bound": round(max(t_tensor, t_hbm) / ms, 4),
            "hbm_gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "hbm_frac": round(nbytes / (ms / 1e3) / 1e9 / hbm_peak, 4)}


def build_dense(device, name, seed=SEED + 3, rule=False):
    """The workload's op; rule=True gives its mask by rule (acefa_flash_attn_ext_gen)."""
    import torch

    import acefa

    B, Hq, Hkv, S_q, S_kv, kind, extra = DENSE_WORKLOADS[name][:7]
    kv = DENSE_WORKLOADS[name][7] if len(DENSE_WORKLOADS[name]) > 7 else "f16"
    hd = DENSE_WORKLOADS[name][8] if len(DENSE_WORKLOADS[name]) > 8 else D
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, Hq, S_q, hd, device=device, generator=g)
    k = torch.randn(B, Hkv, S_kv, hd, device=device, generator=g, dtype=torch.float16)
    v = torch.randn(B, Hkv, S_kv, hd, device=device, generator=g, dtype=torch.float16)
    kv_type = None
    if kv == "bf16":
        k, v = k.bfloat16(), v.bfloat16()
    elif kv == "q8_0":
        k, v, kv_type = acefa.quantize_q8_0(k), acefa.quantize_q8_0(v), acefa.GGML_Q8_0
    mask = None
    if kind is not None:
        qi = torch.arange(S_q, device=device)[:, None]
        kj = torch.arange(S_kv, device=device)[None, :]
        if kind == "causal":
            vis = kj <= qi
        elif kind == "window":
            vis = (qi - kj).abs() <= extra
        else:
            vis = (kj < extra).expand(S_q, S_kv)
        mask = torch.where(vis, 0.0, float("-inf")).half().reshape(1, 1, S_q, S_kv).contiguous()
    if rule and kind is not None:
        mg = {"causal": lambda: acefa.mask_gen(acefa.MASK_CAUSAL, pos0=[S_kv - S_q] * B),
              "window": lambda: acefa.mask_gen(acefa.MASK_WINDOW, window=extra),
              "padding": lambda: acefa.mask_gen(acefa.MASK_PADDING, lens=[extra] * B)}[kind]()
        op = acefa.Op(q, k, v, mask_gen=mg, kv_type=kv_type, scale=hd ** -0.5)
    else:
        op = acefa.Op(q, k, v, mask=mask, kv_type=kv_type, scale=hd ** -0.5)
    flops = 4 * hd * dense_pairs(S_q, S_kv, kind, extra) * Hq * B
    return op, flops


def time_dense(device, stream, name, iters=100, warmup=3, rule=False):
    """One dense op captured in a CUDA graph, `iters` replays timed with CUDA
    events on the launching stream.  An op whose bytes exceed twice the L2 is
    timed as one block of back-to-back replays; a smaller one gets a 256 MB
    L2-flushing write before every replay, outside its own event pair, so no
    replay finds its inputs in L2."""
    import torch

    import acefa

    op, flops = build_dense(device, name, rule=rule)
    flush = dense_bytes(name, rule) < 2 * L2_BYTES
    with torch.cuda.stream(stream):
        op(stream=stream)
        path = acefa.last_path()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            op(stream=stream)
        for _ in range(warmup):
            graph.replay()
        if flush:
            scrub = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
            for a, b in ev:
                scrub.zero_()
                a.record(stream)
                graph.replay()
                b.record(stream)
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in ev) / iters
            del scrub
        else:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(iters):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / iters
    del graph, op
    return {"ms": round(ms, 4), "tflops": round(flops / (ms / 1e3) / 1e12, 1), "gflop": round(flops / 1e9, 2),
            "l2": "flushed before every replay" if flush else "inputs larger than twice the L2; no flush",
            "path": "dense tcgen05" if path == 2 else "decode"}


def dense_extras(device, stream, cpu=True):
    """BASELINE configs 3 and 4: each dense workload timed alone (CUDA graph,
    100 replays, L2 flushed between replays of ops smaller than twice the L2),
    with its roofline (tensor bound, measured bf16 burst peak; DRAM traffic of
    one launch from profiles/ncu_traffic.json when captured; `binding`: the
    longer of the tensor and HBM times and the fraction of it achieved), the
    same op through the C ABI with host buffers (e2e), and for the headline
    shapes the CPU port on sampled query rows."""
    peak = read_tflops_peak()
    hbm_peak = read_peaks()[0]
    res = {"peak_tflops": peak, "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst; kernel timed alone)",
           "peak_hbm_gbs": hbm_peak}
    for name in DENSE_WORKLOADS:
        r = time_dense(device, stream, name)
        r["frac_of_peak"] = round(r["tflops"] / peak, 4)
        nbytes = dense_bytes(name)
        r["roofline"] = {"bound": "tensor", "achieved": r["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": r["frac_of_peak"], "traffic": read_traffic(f"fa_dense_kernel_{name}"),
                         "peak_source": "measured bf16_tflops (burst)", "algo_flop_per_launch": int(r["gflop"] * 1e9),
                         "algo_bytes_per_launch": nbytes,
                         "binding": dense_bound(r["gflop"] * 1e9, nbytes, r["ms"], peak, hbm_peak)}
        if name in ("prefill4096", "dit6000", "cross6000", "prefill1024", "dit1500"):
            r["e2e"] = dense_e2e(device, stream, name)
        if cpu and name in DENSE_CPU_SAMPLED:
            r["cpu_baseline"] = dense_cpu_baseline(name)
        res[name] = r
    # the masked workloads again with the mask given by rule (no mask tensor,
    # no classification pass)
    for name, wl in DENSE_WORKLOADS.items():
        if wl[5] is not None and len(wl) == 7:
            r = time_dense(device, stream, name, rule=True)
            r["frac_of_peak"] = round(r["tflops"] / peak, 4)
            r["binding"] = dense_bound(r["gflop"] * 1e9, dense_bytes(name, rule=True), r["ms"], peak, hbm_peak)
            res[name + "_rule"] = r
    return res


def dense_e2e(device, stream, name, iters=5):
    """The dense op through the C ABI with host buffers: per call the pinned
    H2D of Q, K, V (and mask), acefa_flash_attn_ext, the D2H of the output, in
    stream order (the copies cannot overlap a single op's own attention)."""
    import torch

    op, flops = build_dense(device, name)
    host = {k: torch.empty_like(t, device="cpu").pin_memory() for k, t in
            (("q", op.q), ("k", op.k), ("v", op.v), ("m", op.mask)) if t is not None}
    for k, t in (("q", op.q), ("k", op.k), ("v", op.v), ("m", op.mask)):
        if t is not None:
            host[k].copy_(t)
    out_h = torch.empty_like(op.out, device="cpu").pin_memory()
    dev = {"q": op.q, "k": op.k, "v": op.v, "m": op.mask}

    def step():
        for k, h in host.items():
            dev[k].copy_(h, non_blocking=True)
        op(stream=stream)
        out_h.copy_(op.out, non_blocking=True)

    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    h2d = sum(h.numel() * h.element_size() for h in host.values())
    del op
    return {"ms": round(ms, 3), "tflops": round(flops / (ms / 1e3) / 1e12, 1), "h2d_bytes_per_call": int(h2d),
            "d2h_bytes_per_call": int(out_h.numel() * 4), "how": "pinned H2D of Q/K/V/mask, C-ABI call, D2H of "
            "the output, stream-ordered; CUDA events"}


def dense_cpu_baseline(name, rows_per=24, budget_s=1.5):
    """The oracle (ggml-cpu arithmetic) on `rows_per` sampled query rows of the
    workload (all heads and batches, the rows' full key ranges), at nproc and
    at the reference's default of hw/2 threads (src/backend.h:28-31)."""
    import numpy as np

    import oracle

    B, Hq, Hkv, S_q, S_kv, kind, extra = DENSE_WORKLOADS[name][:7]
    rng = np.random.default_rng(SEED + 3)
    rows = np.sort(rng.choice(S_q, rows_per, replace=False))
    q = rng.standard_normal((B, Hq, rows_per, D), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, S_kv, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((B, Hkv, S_kv, D), dtype=np.float32).astype(np.float16)
    m, vis = None, np.full((rows_per,), S_kv)
    if kind is not None:
        j = np.arange(S_kv)[None, :]
        ri = rows[:, None] + (S_kv - S_q)
        ok = {"causal": j <= ri, "window": np.abs(ri - j) <= (extra or 0),
              "padding": np.broadcast_to(j < (extra or 0), (rows_per, S_kv))}[kind]
        vis = ok.sum(1)
        m = np.where(ok, 0.0, -np.inf).astype(np.float16).reshape(1, 1, rows_per, S_kv)
    flops = 4 * D * Hq * B * int(vis.sum())
    out = {}
    for label, th in (("nproc", os.cpu_count()), ("hw2", max(1, (os.cpu_count() or 2) // 2))):
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.flash_attn_ext(q, k, v, m, scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=th)
            n += 1
        out[label] = {"tflops": round(n * flops / (time.perf_counter() - t0) / 1e12, 5), "cores": th}
    return {"value": out["nproc"]["tflops"], "unit": "TFLOP/s", "cores": out["nproc"]["cores"], "kind": "port",
            "hw2": out["hw2"], "sample": f"{rows_per} sampled query rows x {Hq} heads x B={B} over their visible keys; "
                                           "oracle/fa_oracle.c ggml-cpu arithmetic, OpenMP"}


def sharded_dit(device, stream, world, rank, iters=10, warmup=3):
    """BASELINE config 4 (S=6000, B=2, 16 heads) with K/V head groups split over
    the ranks and one NCCL all-gather of the outputs (strong scaling: the total
    work is fixed).  Device time, max over ranks."""
    import torch
    import torch.distributed as dist

    from acefa.dist import MirroredShardedOp, ShardedOp, head_shard

    B, Hq, Hkv, S = 2, 16, 16, 6000
    g = torch.Generator(device=device).manual_seed(SEED + 11)
    sh = head_shard(Hq, Hkv, world, rank)
    hs, hks = sh.hq1 - sh.hq0, sh.hk1 - sh.hk0
    q = torch.randn(B, hs, S, D, device=device, generator=g)
    k = torch.randn(B, hks, S, D, device=device, generator=g, dtype=torch.float16)
    v = torch.randn(B, hks, S, D, device=device, generator=g, dtype=torch.float16)
    op = ShardedOp(q, k, v, None, world)
    mop = MirroredShardedOp(q, k, v, None, world)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            op(stream)
            mop(stream)
        torch.cuda.synchronize()
        dist.barrier()
        ev[0].record(stream)
        for _ in range(iters):
            op.op(stream)
        ev[1].record(stream)
        for _ in range(iters):
            op(stream)
        ev[2].record(stream)
        for _ in range(iters):
            mop(stream)
        ev[3].record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([ev[i].elapsed_time(ev[i + 1]) / iters for i in range(3)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    mop.close()
    del op, mop, q, k, v
    # the same node unsharded on one GPU (every rank alone, no collective): the
    # denominator of the strong-scaling efficiency
    import acefa

    qf = torch.randn(B, Hq, S, D, device=device, generator=g)
    kf = torch.randn(B, Hkv, S, D, device=device, generator=g, dtype=torch.float16)
    vf = torch.randn(B, Hkv, S, D, device=device, generator=g, dtype=torch.float16)
    full = acefa.Op(qf, kf, vf, scale=D ** -0.5)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            full(stream)
        e0.record(stream)
        for _ in range(iters):
            full(stream)
        e1.record(stream)
        torch.cuda.synchronize()
    t1 = torch.tensor([e0.elapsed_time(e1) / iters], device=device)
    dist.all_reduce(t1, op=dist.ReduceOp.MAX)
    t1 = float(t1[0])
    del full, qf, kf, vf
    flops = 4 * D * S * S * Hq * B
    tf = lambda ms: round(flops / (ms / 1e3) / 1e12, 1)  # noqa: E731
    eff = lambda ms: round(t1 / (world * ms), 4)  # noqa: E731
    return {"gpus": world, "ms_one_gpu_unsharded": round(t1, 4), "ms_attention_only": round(float(t[0]), 4),
            "ms_with_nccl_allgather": round(float(t[1]), 4), "ms_p2p_mirrored": round(float(t[2]), 4),
            "tflops_total_nccl_allgather": tf(float(t[1])), "tflops_total_p2p_mirrored": tf(float(t[2])),
            "strong_scaling_efficiency": {"attention_only": eff(float(t[0])),
                                          "nccl_allgather": eff(float(t[1])),
                                          "p2p_mirrored": eff(float(t[2]))},
            "note": "heads sharded by K/V group; full output on every rank either by NCCL "
                    "all_gather_into_tensor + permute, or by the kernel storing its rows into every "
                    "rank's buffer over NVLink (one-element all-reduce as completion barrier); "
                    "efficiency = one GPU's unsharded time / (N x the sharded time)"}


# -------------------------------------------------------------------------
# the end-to-end attention workload of one generation --
# a random-init Qwen3-4B Q8_0 LM (36 layers, Hq 32 / Hkv 8, 8 requests x CFG =
# 16 KV sets) with a 512-token prompt prefilled per set (qw3lm_forward,
# src/qwen3-lm.h:480-621) and 2000 batched decode steps (qw3lm_forward_batch,
# :629-894) whose window n_kv_pad = PAD(kv_len, 256) grows 768 -> 2560 with the
# graph rebuilt at each new window (:496-500, src/pipeline-lm.cpp:427-527);
# then 8 DiT steps x 24 layers of S = 6000 self-attention (128-key sliding
# window on even layers, src/dit.h:400) and cross-attention to 512 text tokens
# (461 valid), B = 2 (CFG), 16 x 128 heads (src/dit-sampler.h:415).  Masks are
# f16 tensors filled the way the reference fills them.  At N GPUs the 16 KV
# sets split N ways (no collective) and the DiT heads split N ways, each
# rank's kernel storing its heads into every rank's output over NVLink, one
# one-element NCCL all-reduce per node as completion barrier (strong scaling:
# the total work is fixed).
C5_LAYERS, C5_SETS, C5_PROMPT, C5_GEN, C5_MAXSEQ = 36, 16, 512, 2000, 2560
C5_DIT_STEPS, C5_DIT_LAYERS, C5_DIT_S, C5_DIT_ENC, C5_DIT_VALID, C5_DIT_WIN = 8, 24, 6000, 512, 461, 128
Q8_ROW = D // 32 * 34


def pad256(n):
    return (n + 255) // 256 * 256


def c5_decode_bytes(sets, kv_len, n_kv_pad):
    """Algorithmic HBM bytes of one batched decode op: the valid K/V rows of
    every (set, kv head) once, Q and O (f32), the mask rows."""
    return sets * HKV * kv_len * Q8_ROW * 2 + sets * HQ * D * 4 * 2 + sets * n_kv_pad * 2


def c5_prefill_flops(S=C5_PROMPT):
    return 4 * D * HQ * S * (S + 1) // 2  # one set, one layer, unmasked (q, k) pairs


def c5_dit_flops(heads=16, B=2):
    full = 4 * D * heads * B * C5_DIT_S * C5_DIT_S
    win = 4 * D * heads * B * dense_pairs(C5_DIT_S, C5_DIT_S, "window", C5_DIT_WIN)
    cross = 4 * D * heads * B * C5_DIT_S * C5_DIT_VALID
    return full, win, cross


def config5(device, stream, world=1, rank=0, gen=C5_GEN):
    """Runs the whole config-5 workload once untimed (warm-up, graph capture)
    and once timed; device time per part, max over ranks."""
    import torch
    import torch.distributed as dist

    import acefa
    from acefa.dist import MirroredShardedOp, head_shard

    sets = C5_SETS // world
    g = torch.Generator(device=device).manual_seed(SEED + 5000 + 7919 * rank)
    # ---- LM: one Q8_0 KV cache per layer, (sets, Hkv, max_seq, 136 B rows)
    caches = []
    for _ in range(C5_LAYERS):
        kf = torch.randn(sets, HKV, C5_MAXSEQ, D, device=device, generator=g, dtype=torch.float16)
        vf = torch.randn(sets, HKV, C5_MAXSEQ, D, device=device, generator=g, dtype=torch.float16)
        caches.append((acefa.quantize_q8_0(kf), acefa.quantize_q8_0(vf)))
        del kf, vf
    # prompt prefill: one op per (layer, set), Q [128, 512, 32] f32, causal mask
    qp = torch.randn(1, HQ, C5_PROMPT, D, device=device, generator=g)
    mp = torch.where(torch.arange(C5_PROMPT, device=device)[None, :] <= torch.arange(C5_PROMPT, device=device)[:, None],
                     0.0, float("-inf")).half().reshape(1, 1, C5_PROMPT, C5_PROMPT).contiguous()
    outp = torch.empty(1, C5_PROMPT, HQ, D, device=device)
    pre_ops = [acefa.Op(qp, k[s:s + 1, :, :C5_PROMPT], v[s:s + 1, :, :C5_PROMPT], mask=mp, out=outp,
                        kv_type=acefa.GGML_Q8_0, scale=D ** -0.5)
               for (k, v) in caches for s in range(sets)]
    pre_path = None
    # decode: per window, one CUDA graph of all its steps (36 ops each); step
    # i's ops read mask slice i of the window's table (0 up to kv_len, -inf after)
    qd = [torch.randn(sets, HQ, 1, D, device=device, generator=g) for _ in range(C5_LAYERS)]
    outd = [torch.empty(sets, 1, HQ, D, device=device) for _ in range(C5_LAYERS)]
    windows = {}
    for t in range(gen):
        kv_len = C5_PROMPT + t + 1
        windows.setdefault(min(pad256(kv_len), C5_MAXSEQ), []).append(kv_len)
    dec_bytes = sum(c5_decode_bytes(sets, kl, w) for w, kls in windows.items() for kl in kls) * C5_LAYERS
    graphs, keep = [], []
    with torch.cuda.stream(stream):
        for w, kls in sorted(windows.items()):
            lens = torch.tensor(kls, device=device)
            tab = torch.where(torch.arange(w, device=device)[None, :] < lens[:, None], 0.0, float("-inf")).half()
            tab = tab[:, None, None, None, :].expand(len(kls), sets, 1, 1, w).contiguous()
            ops = [acefa.Op(qd[l], caches[l][0][:, :, :w], caches[l][1][:, :, :w], mask=tab[0], out=outd[l],
                            kv_type=acefa.GGML_Q8_0, scale=D ** -0.5) for l in range(C5_LAYERS)]
            for op in ops:  # warm-up outside capture (first-call set-up per kernel instance)
                op(stream=stream)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for i in range(len(kls)):
                    ptr = tab[i].data_ptr()
                    for op in ops:
                        op.tm.data = ptr
                        op(stream=stream)
            graphs.append(gr)
            keep.append((tab, ops))
        for op in pre_ops[:2]:
            op(stream=stream)
        pre_path = acefa.last_path()
        pre_graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(pre_graph, stream=stream):
            for op in pre_ops:
                op(stream=stream)
    # ---- DiT: 24 layers of self (window on even layers) + cross attention
    sh = head_shard(16, 16, world, rank)
    hs = sh.hq1 - sh.hq0
    B, S = 2, C5_DIT_S
    qx = torch.randn(B, hs, S, D, device=device, generator=g)
    qi = torch.arange(S, device=device)
    mwin = torch.where((qi[:, None] - qi[None, :]).abs() <= C5_DIT_WIN, 0.0, float("-inf")).half()
    mwin = mwin.reshape(1, 1, S, S).contiguous()
    mpad = torch.where(torch.arange(C5_DIT_ENC, device=device) < C5_DIT_VALID, 0.0, float("-inf")).half()
    mpad = mpad.reshape(1, 1, 1, C5_DIT_ENC).expand(B, 1, S, C5_DIT_ENC).contiguous()
    dit_ops = []
    out1 = torch.empty(B, S, hs, D, device=device) if world == 1 else None
    for l in range(C5_DIT_LAYERS):
        ks = torch.randn(B, hs, S, D, device=device, generator=g, dtype=torch.float16)
        vs = torch.randn(B, hs, S, D, device=device, generator=g, dtype=torch.float16)
        kc = torch.randn(B, hs, C5_DIT_ENC, D, device=device, generator=g, dtype=torch.float16)
        vc = torch.randn(B, hs, C5_DIT_ENC, D, device=device, generator=g, dtype=torch.float16)
        for kk, vv, mm in ((ks, vs, mwin if l % 2 == 0 else None), (kc, vc, mpad)):
            if world == 1:  # the full output directly, no gather
                dit_ops.append(acefa.Op(qx, kk, vv, mask=mm, out=out1, scale=D ** -0.5))
            else:  # each rank's kernel stores its heads into every rank's full output
                dit_ops.append(MirroredShardedOp(qx, kk, vv, mm, world, scale=D ** -0.5))

    def run_dit(steps):
        for _ in range(steps):
            for op in dit_ops:
                op(stream)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    with torch.cuda.stream(stream):
        pre_graph.replay()
        for gr in graphs:
            gr.replay()
        run_dit(1)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev[0].record(stream)
        pre_graph.replay()
        ev[1].record(stream)
        for gr in graphs:
            gr.replay()
        ev[2].record(stream)
        run_dit(C5_DIT_STEPS)
        ev[3].record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])],
                     device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    assert acefa.device_error(stream) == 0
    ms_pre, ms_dec, ms_dit = (float(x) for x in t)
    hbm, _ = read_peaks()
    tf_peak = read_tflops_peak()
    pre_fl = c5_prefill_flops() * C5_LAYERS * C5_SETS
    full, win, cross = c5_dit_flops()
    dit_fl = C5_DIT_STEPS * (C5_DIT_LAYERS // 2) * (full + win) + C5_DIT_STEPS * C5_DIT_LAYERS * cross
    dec_total = dec_bytes * world
    for op in dit_ops:
        if world > 1:
            op.close()
    del graphs, pre_graph, keep, pre_ops, dit_ops, caches
    torch.cuda.empty_cache()
    return {
        "gpus": world, "wall_ms": round(ms_pre + ms_dec + ms_dit, 2),
        "prefill": {"ms": round(ms_pre, 3), "ops": C5_LAYERS * C5_SETS, "gflop": round(pre_fl / 1e9, 1),
                    "tflops": round(pre_fl / (ms_pre / 1e3) / 1e12, 1),
                    "frac_of_bf16_peak": round(pre_fl / (ms_pre / 1e3) / 1e12 / tf_peak, 4),
                    "path": "dense tcgen05" if pre_path == 2 else "split-KV decode kernel"},
        "decode": {"ms": round(ms_dec, 2), "steps": gen, "ops": gen * C5_LAYERS,
                   "windows": sorted(windows), "gb": round(dec_total / 1e9, 2),
                   "gbs": round(dec_total / (ms_dec / 1e3) / 1e9, 1),
                   "frac_of_hbm_peak": round(dec_total / (ms_dec / 1e3) / 1e9 / hbm, 4),
                   "us_per_op": round(ms_dec * 1e3 / (gen * C5_LAYERS), 2)},
        "dit": {"ms": round(ms_dit, 2), "steps": C5_DIT_STEPS, "layers": C5_DIT_LAYERS,
                "tflop": round(dit_fl / 1e12, 2), "tflops": round(dit_fl / (ms_dit / 1e3) / 1e12, 1),
                "frac_of_bf16_peak": round(dit_fl / (ms_dit / 1e3) / 1e12 / tf_peak, 4),
                "assembly": ("kernel stores its heads into every rank's output over NVLink + one-element "
                             "NCCL all-reduce per op") if world > 1 else "single GPU"},
        "note": "device time per part (CUDA events, max over ranks); decode bytes count valid K/V rows; "
                "f16 masks filled like the reference's; LM KV sets and DiT heads split over the GPUs",
    }


def read_tflops_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0


def config5_cpu_baseline(budget_s=6.0, threads=None):
    """The reference operator's CPU arithmetic (oracle, ggml-cpu mode) on bounded
    samples of config 5: one batched Q8_0 decode op at a mid window and a slice of
    DiT query rows; the whole workload's CPU time is estimated from their rates."""
    import numpy as np

    import oracle

    threads = threads or os.cpu_count()
    rng = np.random.default_rng(SEED + 5)
    kv_len, w = 1536, 1536
    q = rng.standard_normal((C5_SETS, HQ, 1, D), dtype=np.float32)
    kq = oracle.quantize_q8_0(rng.standard_normal((C5_SETS, HKV, w, D), dtype=np.float32))
    vq = oracle.quantize_q8_0(rng.standard_normal((C5_SETS, HKV, w, D), dtype=np.float32))
    m = np.zeros((C5_SETS, 1, 1, w), np.float16)
    args = dict(scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, k_type=oracle.GGML_Q8_0, v_type=oracle.GGML_Q8_0,
                d=D, dv=D, nthreads=threads)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s / 2 or n == 0:
        oracle.flash_attn_ext(q, kq, vq, m, **args)
        n += 1
    dec_gbs = n * c5_decode_bytes(C5_SETS, kv_len, w) / (time.perf_counter() - t0) / 1e9
    rows = 64
    qd = rng.standard_normal((2, 16, rows, D), dtype=np.float32)
    kd = rng.standard_normal((2, 16, C5_DIT_S, D), dtype=np.float32).astype(np.float16)
    vd = rng.standard_normal((2, 16, C5_DIT_S, D), dtype=np.float32).astype(np.float16)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s / 2 or n == 0:
        oracle.flash_attn_ext(qd, kd, vd, None, scale=D ** -0.5, mode=oracle.MODE_GGML_CPU, nthreads=threads)
        n += 1
    dit_tflops = n * 4 * D * 16 * 2 * rows * C5_DIT_S / (time.perf_counter() - t0) / 1e12
    windows = {}
    for t in range(C5_GEN):
        kl = C5_PROMPT + t + 1
        windows.setdefault(pad256(kl), []).append(kl)
    dec_bytes = sum(c5_decode_bytes(C5_SETS, kl, w) for w, kls in windows.items() for kl in kls) * C5_LAYERS
    full, win, cross = c5_dit_flops()
    dit_fl = C5_DIT_STEPS * (C5_DIT_LAYERS // 2) * (full + win) + C5_DIT_STEPS * C5_DIT_LAYERS * cross
    pre_fl = c5_prefill_flops() * C5_LAYERS * C5_SETS
    est_s = dec_bytes / (dec_gbs * 1e9) + (dit_fl + pre_fl) / (dit_tflops * 1e12)
    return {"decode_gbs": round(dec_gbs, 2), "dense_tflops": round(dit_tflops, 4), "cores": threads,
            "kind": "port", "estimated_wall_s": round(est_s, 1),
            "sample": f"one 16-set Q8_0 decode op at window {w} and {rows} query rows x 16 heads x B=2 of "
                      f"DiT self-attention over {C5_DIT_S} keys, oracle/fa_oracle.c ggml-cpu arithmetic, "
                      f"OpenMP; the workload's CPU time is estimated from these two rates"}


def run_dense_workload(args):
    """--workload <dense name>: time one dense op (also the ncu profiling case);
    --workload dit6000_prologue: the DiT layer with its QK-norm + RoPE prologue."""
    import torch

    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    stream = torch.cuda.Stream(device=device)
    if args.workload == "dit6000_prologue":
        emit({"workload": args.workload, **dit_prologue(device, stream, iters=args.steps)})
        return 0
    if args.workload == "config5":
        emit({"workload": args.workload, **config5(device, stream, gen=args.c5_gen)})
        return 0
    if args.workload == "cfg_combine":
        emit({"workload": args.workload, **cfg_combine_step(device, stream, iters=args.steps)})
        return 0
    if args.workload == "config1":
        # 64 distinct Qwen3-0.6B decode ops back to back
        # (also the ncu profiling case of the op)
        import acefa

        g = torch.Generator(device=device).manual_seed(42 + 1000)
        ops = []
        for _ in range(64):
            q = torch.randn(1, 16, 1, D, device=device, generator=g)
            k = torch.randn(1, 8, 2048, D, device=device, generator=g, dtype=torch.float16)
            v = torch.randn(1, 8, 2048, D, device=device, generator=g, dtype=torch.float16)
            ops.append(acefa.Op(q, k, v, mask=torch.zeros(1, 1, 1, 2048, device=device, dtype=torch.float16),
                                scale=D ** -0.5))
        graph = time_graph(ops, args.steps, args.warmup, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.steps * len(ops))
        emit({"workload": "config1", "us_per_op": round(us, 2), "gbs": round(8_409_088 / (us / 1e6) / 1e9, 1)})
        return 0
    r = time_dense(device, stream, args.workload, iters=args.steps, warmup=args.warmup, rule=args.mask_rule)
    emit({"workload": args.workload, "mask_rule": bool(args.mask_rule), **r})
    return 0


_JSON_FD = None


def claim_stdout():
    """Keep stdout for the one JSON line: libraries that print on fd 1 (NCCL's
    version banner under torchrun, for one) are sent to stderr instead."""
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)


def emit(obj):
    data = (json.dumps(obj) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def main():
    claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers per step (36 = the headline stack)")
    ap.add_argument("--kv", default="f16", choices=["f16", "q8_0"])
    ap.add_argument("--workload", default="decode4b",
                    help="decode4b (headline), config1, config5, dit6000_prologue, cfg_combine, or one dense op: " +
                         ", ".join(DENSE_WORKLOADS))
    ap.add_argument("--no-config5", action="store_true", help="skip the config-5 end-to-end workload extra")
    ap.add_argument("--c5-gen", type=int, default=C5_GEN, help="config-5 decode steps (2000 = the BASELINE workload)")
    ap.add_argument("--mask-rule", action="store_true",
                    help="dense workload: give the mask by rule (acefa_flash_attn_ext_gen) instead of a tensor")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "decode4b":
        return run_dense_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
