"""Benchmark of the compressed Butterfly attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: one compressed-attention layer at T=32768,
Hq 8 / Hkv 2, head_dim 128, block 128, window 64, bf16, run once per causal_shift stage
0..7 (layers 0..7, partner offsets 1..128).  One step = those 8 layer passes, each on
its own seeded N(0,1) Q/K/V (8 x 100.7 MB resident inputs > 126 MB L2), each pass =
mean-pool compressor for K and V + the tcgen05 prefill kernel.
metric = prefill layer-tokens/s = 8 * T * n_gpus / step time (weak scaling: every rank
runs its own sequence — batch sharding, no data-path collective).

Also measured: BASELINE config 5 decode (64 sequences pre-filled to 65536 tokens in the
two-pool cache, 128 fused append+close+attend steps replayed from a CUDA graph) as
decode us/step and HBM GB/s, reported under "decode".

--impl reference times the reference's CPU algorithm (the PyTorch-CPU port in oracle/,
fp32, all host threads) on one layer pass of the same workload per step, rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

T, HQ, HKV, DH, BS, W = 32768, 8, 2, 128, 128, 64
LAYERS = list(range(8))
L2_BYTES = 126 * 2**20


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
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
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return ws, rank, local


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        try:
            return int(ids[local])
        except (ValueError, IndexError):
            return local
    return local


# ----------------------------------------------------------------------------- prefill (c2)
def _layouts(seq_len):
    import butterfly_b200 as bb
    return [bb.build_block_butterfly_layout(seq_len=seq_len, block_size=BS, num_key_value_heads=HKV,
                                            num_key_value_groups=HQ // HKV, layer_idx=l, local_window_blocks=1,
                                            sink_count=1, partner_count=1, partner_rule="causal_shift")
            for l in LAYERS]


def prefill_bytes_per_launch() -> int:
    """Algorithmic HBM bytes of one prefill-kernel launch: read Q, K, V and the routed block
    means, write O (bf16).  Summaries are read once per (block, KV head)."""
    N = -(-T // BS)
    return 2 * DH * T * (HQ + 2 * HKV + HQ) + 2 * 2 * HKV * N * DH


def compress_bytes_per_pair() -> int:
    N = -(-T // BS)
    return 2 * (2 * DH * T * HKV) + 2 * (2 * DH * N * HKV)


def run_prefill(dev, seed, steps, warmup, sampler):
    from butterfly_b200.attention import block_mean_summaries_kv, prefill_attention_into, route_for
    g = torch.Generator(device=dev).manual_seed(seed)
    ins = []
    for _ in LAYERS:
        q = torch.randn(1, HQ, T, DH, device=dev, generator=g).bfloat16()
        k = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
        v = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
        ins.append((q, k, v))
    lays = _layouts(T)
    routes = [route_for(l, dev)[0] for l in lays]
    N = lays[0].num_blocks
    ks = [torch.empty(1, HKV, N, DH, device=dev, dtype=torch.bfloat16) for _ in LAYERS]
    vs = [torch.empty_like(x) for x in ks]
    outs = [torch.empty(1, T, HQ, DH, device=dev, dtype=torch.bfloat16).transpose(1, 2) for _ in LAYERS]
    scale = 1.0 / math.sqrt(DH)
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in LAYERS] for _ in range(steps)]

    def step(si=None):
        for i in range(len(LAYERS)):
            q, k, v = ins[i]
            if si is not None:
                ev[si][i][0].record()
            block_mean_summaries_kv(k, v, seq_len=T, block_size=BS, num_blocks=N, k_out=ks[i], v_out=vs[i])
            if si is not None:
                ev[si][i][1].record()
            prefill_attention_into(q, k, v, ks[i], vs[i], outs[i], None, routes[i], W, scale)
            if si is not None:
                ev[si][i][2].record()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    return step, ev, ins, lays


def run_e2e(dev, lays, ins, steps):
    """Public API from pinned host buffers: H2D of Q/K/V, the call, D2H of the output.

    Layers are pipelined over three streams (copy-in, compute, copy-out) so that the
    inputs of layer i+1 cross PCIe while layer i computes and layer i-1's output copies
    back; each step still moves every layer's inputs in and its output out."""
    import butterfly_b200 as bb
    host = [tuple(x.cpu().pin_memory() for x in t) for t in ins]
    outh = [torch.empty(1, HQ, T, DH, dtype=torch.bfloat16).pin_memory() for _ in LAYERS]
    devin = [tuple(torch.empty_like(x, device=dev) for x in t) for t in host]
    h2d = sum(x.numel() * x.element_size() for t in host for x in t)
    d2h = sum(x.numel() * x.element_size() for x in outh)
    s_in, s_cmp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    n = len(LAYERS)
    in_ready = [torch.cuda.Event() for _ in LAYERS]
    used = [torch.cuda.Event() for _ in LAYERS]      # compute of layer i done reading its inputs
    out_ready = [torch.cuda.Event() for _ in LAYERS]
    for e in used:
        e.record(s_cmp)

    def step():
        for i in range(n):
            s_in.wait_event(used[i])  # the previous step's layer i finished with devin[i]
            with torch.cuda.stream(s_in):
                for d, h in zip(devin[i], host[i]):
                    d.copy_(h, non_blocking=True)
                in_ready[i].record(s_in)
            s_cmp.wait_event(in_ready[i])
            with torch.cuda.stream(s_cmp):
                q, k, v = devin[i]
                y = bb.butterfly_compressed_attention(q, k, v, layout=lays[i], local_window_tokens=W)
                used[i].record(s_cmp)
                out_ready[i].record(s_cmp)
            s_out.wait_event(out_ready[i])
            with torch.cuda.stream(s_out):
                y.record_stream(s_out)
                outh[i].copy_(y, non_blocking=True)

    def run(k):
        cur = torch.cuda.current_stream(dev)
        for s_ in (s_in, s_cmp, s_out):
            s_.wait_stream(cur)
        for _ in range(k):
            step()
        for s_ in (s_in, s_cmp, s_out):
            cur.wait_stream(s_)

    run(1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run(steps)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return ms, h2d, d2h


# ----------------------------------------------------------------------------- decode (c5)
DEC_B, DEC_CTX, DEC_STEPS, DEC_CHUNK = 64, 65536, 128, 4096


def decode_bytes_per_step() -> int:
    """Per step, per (sequence, KV head): raw window K+V (W rows), <=2 routed summaries (K+V),
    the query heads and outputs, the appended token (read + ring write) and the amortised
    block close (BS rows of K and V read once every BS steps, plus the summary writes)."""
    row = DH * 2
    g = HQ // HKV
    per = 2 * W * row + 2 * 2 * row + 2 * g * row + 2 * 2 * row + (2 * BS * row + 2 * row) / BS
    return int(per * DEC_B * HKV)


def run_decode(dev, seed, reps, warmup):
    import butterfly_b200 as bb
    from butterfly_b200.cache import CompressedKVCache
    g = torch.Generator(device=dev).manual_seed(seed)
    cache = CompressedKVCache(block_size=BS, local_window_tokens=W, max_kv_size=DEC_CTX + DEC_STEPS,
                              max_chunk_size=DEC_CHUNK)
    for c0 in range(0, DEC_CTX, DEC_CHUNK):
        k = torch.randn(DEC_B, HKV, DEC_CHUNK, DH, device=dev, generator=g).bfloat16()
        v = torch.randn(DEC_B, HKV, DEC_CHUNK, DH, device=dev, generator=g).bfloat16()
        cache.append(k, v)
    q = torch.randn(DEC_STEPS, DEC_B, HQ, 1, DH, device=dev, generator=g).bfloat16()
    kn = torch.randn(DEC_STEPS, DEC_B, HKV, 1, DH, device=dev, generator=g).bfloat16()
    vn = torch.randn(DEC_STEPS, DEC_B, HKV, 1, DH, device=dev, generator=g).bfloat16()
    lays = [bb.build_block_butterfly_layout(seq_len=DEC_CTX + s + 1, block_size=BS, num_key_value_heads=HKV,
                                            num_key_value_groups=HQ // HKV, layer_idx=3, local_window_blocks=1,
                                            sink_count=1, partner_count=1, partner_rule="causal_shift")
            for s in range(DEC_STEPS)]
    torch.cuda.synchronize()
    counters = (cache.offset, cache.summary_offset, cache.summary_count, cache.tail_size)
    s = torch.cuda.Stream(device=dev)
    graph = torch.cuda.CUDAGraph()
    outs = []
    with torch.cuda.stream(s):
        # one eager pass on the capture stream (kernel attributes, allocator warm-up)
        for i in range(DEC_STEPS):
            cache.decode_step(q[i], kn[i], vn[i], lays[i])
        torch.cuda.synchronize()
        cache.offset, cache.summary_offset, cache.summary_count, cache.tail_size = counters
        with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
            for i in range(DEC_STEPS):
                outs.append(cache.decode_step(q[i], kn[i], vn[i], lays[i]))
    torch.cuda.synchronize()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * DEC_STEPS)
    return us, cache


# ----------------------------------------------------------------------------- CPU legs
def cpu_port_layer_seconds(layer: int, seed: int = 0) -> float:
    """One config-2 layer pass of the reference's CPU algorithm (oracle/torch_port.py, fp32)."""
    from oracle import topology as ot
    from oracle import torch_port
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, HQ, T, DH, generator=g)
    k = torch.randn(1, HKV, T, DH, generator=g)
    v = torch.randn(1, HKV, T, DH, generator=g)
    nb = ot.block_neighbors_table(-(-T // BS), layer, local_window_blocks=1, sink_count=1, partner_count=1,
                                  partner_rule="causal_shift")
    t0 = time.perf_counter()
    torch_port.prefill(q, k, v, nb, block_size=BS, window=W)
    return time.perf_counter() - t0


def cpu_baseline(budget_s: float = 12.0):
    torch.set_num_threads(os.cpu_count() or 1)
    cpu_port_layer_seconds(0)  # warm-up
    times, t_start, i = [], time.perf_counter(), 0
    while time.perf_counter() - t_start < budget_s and i < 64:
        times.append(cpu_port_layer_seconds(LAYERS[i % len(LAYERS)], seed=i))
        i += 1
    per = statistics.median(times)
    return {"value": round(T / per, 1), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} layer passes (layers 0-7 cycling) of config 2 at full T={T}, fp32, "
                      f"median {per:.3f} s per pass; oracle/torch_port.py restates the reference's "
                      f"CPU algorithm (gather + masked SDPA)"}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    for i in range(args.warmup):
        cpu_port_layer_seconds(LAYERS[i % len(LAYERS)], seed=i)
    times = [cpu_port_layer_seconds(LAYERS[i % len(LAYERS)], seed=100 + i) for i in range(args.steps)]
    per = sum(times) / len(times)
    val = T / per
    line = {
        "impl": "reference", "metric": "prefill_layer_tok_per_s", "value": round(val, 1), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": "config2: one compressed layer pass, T=32768, Hq8/Hkv2, dh128, BS128, W64, "
                               "causal_shift stages 0-7 cycling; one pass per step (bounded CPU sample)"},
        "cpu_baseline": {"value": round(val, 1), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": "one config-2 layer pass per step, fp32, oracle/torch_port.py"},
        "e2e": {"value": round(val, 1), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _traffic_from_profiles():
    p = os.path.join(ROOT, "profiles", "prefill_c2_ncu.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


def prefill_trace(dev):
    """Per-unit pipeline timeline of one config-2 prefill launch (globaltimer stamps)."""
    import ctypes
    from butterfly_b200 import _lib
    from butterfly_b200.attention import block_mean_summaries, prefill_attention_into, route_for
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(1, HQ, T, DH, device=dev, generator=g).bfloat16()
    k = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
    v = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
    lay = _layouts(T)[5]
    r = route_for(lay, dev)[0]
    N = lay.num_blocks
    ks = block_mean_summaries(k, seq_len=T, block_size=BS, num_blocks=N)
    vs = block_mean_summaries(v, seq_len=T, block_size=BS, num_blocks=N)
    out = torch.empty(1, T, HQ, DH, device=dev, dtype=torch.bfloat16).transpose(1, 2)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    buf = torch.zeros(nsm * 64 * 16, dtype=torch.int64, device=dev)
    for _ in range(3):
        prefill_attention_into(q, k, v, ks, vs, out, None, r, W, 1 / math.sqrt(DH))
    _lib.lib().bna_set_prefill_trace(ctypes.c_void_p(buf.data_ptr()))
    prefill_attention_into(q, k, v, ks, vs, out, None, r, W, 1 / math.sqrt(DH))
    torch.cuda.synchronize()
    _lib.lib().bna_set_prefill_trace(None)
    tr = buf.view(nsm, 64, 16).cpu().numpy().astype("int64")
    t0 = tr[:, :, :16][tr[:, :, :16] > 0].min()
    names = ["q_issued", "k_issued", "prod_full", "mma_qk", "mma_pv", "smx_s", "smx_p", "smx_o", "smx_done",
             "-", "-", "-", "-", "-", "-", "v_full"]
    for cta in (0,):
        print(f"cta {cta} (us from kernel start)")
        for i in range(16):
            row = tr[cta, i, :16]
            if row.max() == 0:
                break
            print(f"  unit {i:2d}: " + " ".join(f"{n}={(x - t0) / 1000:7.2f}" for n, x in zip(names, row) if n != "-" and x > 0))
    end = tr[:, :, 8].max()
    print(f"kernel span from first stamp: {(end - t0) / 1000:.2f} us")


def profile_case(kind: str):
    """Small, self-terminating case for ncu captures (a few hundred MB on the device)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if kind == "prefill-trace":
        prefill_trace(dev)
        return
    if kind == "prefill":
        import butterfly_b200 as bb
        from butterfly_b200.attention import block_mean_summaries, prefill_attention_into, route_for
        Tp = 65536  # 201 MB of Q/K/V: larger than L2
        g = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(1, HQ, Tp, DH, device=dev, generator=g).bfloat16()
        k = torch.randn(1, HKV, Tp, DH, device=dev, generator=g).bfloat16()
        v = torch.randn(1, HKV, Tp, DH, device=dev, generator=g).bfloat16()
        lay = bb.build_block_butterfly_layout(seq_len=Tp, block_size=BS, num_key_value_heads=HKV,
                                              num_key_value_groups=HQ // HKV, layer_idx=5, local_window_blocks=1,
                                              sink_count=1, partner_count=1, partner_rule="causal_shift")
        r = route_for(lay, dev)[0]
        N = lay.num_blocks
        ks = block_mean_summaries(k, seq_len=Tp, block_size=BS, num_blocks=N)
        vs = block_mean_summaries(v, seq_len=Tp, block_size=BS, num_blocks=N)
        out = torch.empty(1, Tp, HQ, DH, device=dev, dtype=torch.bfloat16).transpose(1, 2)
        for _ in range(3):
            prefill_attention_into(q, k, v, ks, vs, out, None, r, W, 1 / math.sqrt(DH))
        torch.cuda.synchronize()
    else:
        run_decode(dev, 0, reps=1, warmup=1)
    torch.cuda.synchronize()
    print("profile case done", flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile-case", choices=["prefill", "decode", "prefill-trace"], default=None,
                    help="small case for ncu: warm-up, then exactly one launch of the kernel")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    args.warmup = max(args.warmup, 3)
    ws, rank, local = _dist() if args.impl == "ours" else (int(os.environ.get("WORLD_SIZE", "1")),
                                                           int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm_peak, tc_peak, peak_kind = _peaks()

    step, ev, ins, lays = run_prefill(dev, 1000 + rank, args.steps, args.warmup, None)
    # The timed step (8 layers x compressor + prefill) replays from a CUDA graph, so the
    # Python/ctypes cost of 16 library calls per step stays off the device timeline.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step()
    for _ in range(args.warmup):
        graph.replay()
    sampler = ClockSampler(_gpu_index(local))
    sampler.start()
    _barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for si in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    # per-kernel durations (roofline): the same steps launched eagerly, each kernel
    # bracketed by events on its stream.  A device-side sleep queued first lets the host
    # enqueue the whole pass before the GPU reaches it, so no launch waits on the host.
    torch.cuda._sleep(int(2e8))
    for si in range(args.steps):
        step(si)
    torch.cuda.synchronize()
    _barrier(ws)
    clocks = sampler.stop()
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = _max_over_ranks(ms_local, ws)
    pf = [ev[s][i][1].elapsed_time(ev[s][i][2]) for s in range(args.steps) for i in range(len(LAYERS))]
    cp = [ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps) for i in range(len(LAYERS))]
    pf_ms = sum(pf) / len(pf)
    cp_ms = sum(cp) / len(cp)
    value = len(LAYERS) * T * ws / (ms / 1000.0)

    e2e_ms, h2d, d2h = run_e2e(dev, lays, ins, max(1, min(3, args.steps)))
    e2e_ms = _max_over_ranks(e2e_ms, ws)
    e2e_val = len(LAYERS) * T * ws / (e2e_ms / 1000.0)

    decode = None
    if not args.no_decode:
        del ins
        torch.cuda.empty_cache()
        us, cache = run_decode(dev, 2000 + rank, reps=10, warmup=3)
        us = _max_over_ranks(us, ws)
        gbs = decode_bytes_per_step() / (us * 1e-6) / 1e9
        decode = {"config": "config5: B=64 sequences x 65536 pre-filled tokens (two-pool cache, chunks of 4096), "
                            "Hq8/Hkv2, dh128, BS128, W64; 128 fused append+close+attend steps, CUDA-graph replay",
                  "us_per_step": round(us, 3), "sequences_per_step": DEC_B * ws,
                  "us_per_token_per_sequence": round(us, 3),
                  "algorithmic_bytes_per_step": decode_bytes_per_step(),
                  "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 4),
                  "retained_kv_bytes_per_layer": cache.nbytes,
                  "dense_kv_bytes_per_layer": 2 * DEC_B * HKV * (DEC_CTX + DEC_STEPS) * DH * 2}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_baseline()

    pf_bytes = prefill_bytes_per_launch()
    achieved = pf_bytes / (pf_ms / 1000.0) / 1e9
    line = {
        "metric": "prefill_layer_tok_per_s", "value": round(value, 1), "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) Q/K/V per layer (BASELINE config 2 shapes)",
        "config": {"workload": "config2: compressed-attention layer, T=32768, Hq8/Hkv2, dh128, BS128, W64, "
                               "causal_shift layers 0-7 (stages 0-7) per step; compressor + tcgen05 prefill",
                   "global_batch": ws, "seq_len": T, "parallelism": f"batch-sharded x{ws} (one sequence per GPU)",
                   "l2": f"inputs larger than L2: {len(LAYERS)} distinct layer inputs, "
                         f"{len(LAYERS) * 2 * DH * T * (HQ + 2 * HKV) / 2**20:.0f} MiB per step > 126 MiB L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": _traffic_from_profiles(),
                     "kernel": "prefill_sm100_kernel", "bytes_per_launch": pf_bytes,
                     "ms_per_launch": round(pf_ms, 5), "peak_kind": f"{peak_kind} (hbm_gbs burst copy)",
                     "compressor_pair_ms": round(cp_ms, 5),
                     "compressor_gbs": round(compress_bytes_per_pair() / (cp_ms / 1000.0) / 1e9, 1)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_val, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "butterfly_b200.butterfly_compressed_attention from pinned host buffers; layers "
                        "pipelined over copy-in / compute / copy-out streams"},
        "gpu_launches": args.steps * len(LAYERS) * 2,
        "timing": "ms_per_step from CUDA-graph replays of the step; kernel ms from an eager pass with events",
        "clocks": clocks,
        "decode": decode,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
