"""Benchmark of the compressed Butterfly attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload ("model-128k"): a 0.8B-class Qwen3.5 decoder with random-init weights
(seed 1, bf16): 24 layers, hidden 1024, 8 query / 2 KV heads, head_dim 128, SwiGLU 3584,
vocab 151936, every layer swapped onto compressed Butterfly attention (block 128, window
64) through ``swap_qwen_attention_with_butterfly_cuda``.  One step = one prefill of a
131072-token prompt of uniform random token ids (``logits_to_keep=1``) into a fresh
two-pool cache.  metric = prefill tok/s = T * n_gpus / step time (weak scaling: one
sequence per GPU, no data-path collective).  After the timed prefills, 32 greedy decode
steps from the prefilled cache are captured in a CUDA graph and timed as decode us/token.

Also reported in the same line:
  layer        one attention layer at T=32768 (Hq8/Hkv2), run once per causal_shift stage
               0..7: compressor + tcgen05 prefill, kernel-level HBM roofline;
  decode_batched  64 sequences pre-filled to 65536 tokens in the two-pool cache, 128 fused
               append+close+attend steps replayed from a CUDA graph (decode us/step, HBM);
  cpu_baseline the reference's CPU algorithm (PyTorch, fp32, all host threads).

--impl reference times the reference's CPU algorithm (oracle/ restatement, fp32, all host
threads) on the same model workload: one full-length decoder layer per step, the model
time being 24 such layers (rank 0 only); it also times the reference algorithm on the GPU
(gather + masked SDPA in bf16) as a same-box comparison.
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

# attention-layer workload (one layer, stages 0..7)
T, HQ, HKV, DH, BS, W = 32768, 8, 2, 128, 128, 64
LAYERS = list(range(8))
L2_BYTES = 126 * 2**20

# model workload (0.8B-class decoder at 128k)
MODEL = dict(hidden=1024, layers=24, heads=8, kv_heads=2, head_dim=128, inter=3584, vocab=151936)
MODEL_T = 131072
MODEL_DECODE = 32
MODEL_CHUNK = 4096  # two-pool cache max_chunk_size (the reference harness's kv_step default)


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


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


def _events(n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


# ----------------------------------------------------------------------------- model (128k)
def model_config(spec=MODEL):
    from transformers import Qwen3_5TextConfig
    return Qwen3_5TextConfig(hidden_size=spec["hidden"], intermediate_size=spec["inter"],
                             num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
                             num_key_value_heads=spec["kv_heads"], head_dim=spec["head_dim"],
                             vocab_size=spec["vocab"], layer_types=["full_attention"] * spec["layers"],
                             max_position_embeddings=max(262144, MODEL_T + 4096))


def build_model(dev, seed: int, spec=MODEL, swap: bool = True):
    """Random-init Qwen3.5 decoder in bf16 on ``dev``; every layer swapped when ``swap``."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from butterfly_b200.integrations import qwen_torch as qt
    qt.patch_qwen35_full_attention_decode()
    torch.manual_seed(seed)
    with torch.device(dev):
        m = Qwen3_5ForCausalLM(model_config(spec))
    m = m.to(torch.bfloat16).eval()
    if swap:
        qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    return m


def model_linear_flops_per_token(spec=MODEL) -> int:
    h, hq, hk, d, I = spec["hidden"], spec["heads"], spec["kv_heads"], spec["head_dim"], spec["inter"]
    per_layer = h * (2 * hq * d) + 2 * h * hk * d + hq * d * h + 3 * h * I
    return 2 * per_layer * spec["layers"]


def attention_valid_keys(seq_len: int, layer: int, block_size: int = BS, window: int = W) -> int:
    """Sum over queries of the keys each attends to (raw window + routed summaries), from the
    selection the kernels use (host dump of the same code)."""
    import numpy as np

    import butterfly_b200 as bb
    from butterfly_b200.attention import prefill_selection
    lay = bb.build_block_butterfly_layout(seq_len=seq_len, block_size=block_size, num_key_value_heads=1,
                                          num_key_value_groups=1, layer_idx=layer, local_window_blocks=1,
                                          sink_count=1, partner_count=1, partner_rule="causal_shift")
    _, _, cnt = prefill_selection(lay, seq_len, window)
    rows = np.minimum(block_size, seq_len - np.arange(len(cnt)) * block_size)
    raw = sum(min(q + 1, window) for q in range(window)) + max(0, seq_len - window) * window
    return int(raw + int((cnt.astype(np.int64) * rows).sum()))


def model_prefill_flops(seq_len: int, spec=MODEL) -> int:
    """Algorithmic FLOPs of one prefill: every linear layer (2 per MAC) for every token,
    the attention score and value products over the selected keys (4 * dh per query head
    and key), and the lm_head for the one kept position."""
    att = sum(4 * spec["head_dim"] * spec["heads"] * attention_valid_keys(seq_len, l) for l in range(spec["layers"]))
    return model_linear_flops_per_token(spec) * seq_len + att + 2 * spec["hidden"] * spec["vocab"]


def model_decode_bytes_per_token(ctx: int, spec=MODEL) -> int:
    """HBM bytes one decode token must move: every weight but the embedding table (bf16),
    one embedding row, and per layer the attention's K/V window and summaries."""
    h, hq, hk, d, I, V = (spec[x] for x in ("hidden", "heads", "kv_heads", "head_dim", "inter", "vocab"))
    lin = spec["layers"] * (h * 2 * hq * d + 2 * h * hk * d + hq * d * h + 3 * h * I + 2 * h + 2 * d)
    weights = 2 * (lin + h + h * V) + 2 * h
    kv = spec["layers"] * hk * (2 * W + 2 * 2) * d * 2
    return int(weights + kv)


class ModelBench:
    def __init__(self, dev, rank: int):
        from transformers import DynamicCache

        from butterfly_b200.integrations import qwen_torch as qt
        self.qt, self.DynamicCache = qt, DynamicCache
        self.dev = dev
        self.model = build_model(dev, seed=1)
        g = torch.Generator().manual_seed(1000 + rank)
        self.ids_host = torch.randint(0, MODEL["vocab"], (1, MODEL_T), generator=g).pin_memory()
        self.ids = self.ids_host.to(dev)
        self.logits_host = torch.empty((1, 1, MODEL["vocab"]), dtype=torch.bfloat16).pin_memory()

    def new_cache(self):
        return self.qt.make_compressed_cache(self.model, self.DynamicCache(config=self.model.config),
                                             max_kv_size=MODEL_T + MODEL_DECODE, max_chunk_size=MODEL_CHUNK)

    @torch.no_grad()
    def prefill(self, ids=None):
        cache = self.new_cache()
        out = self.model(input_ids=self.ids if ids is None else ids, past_key_values=cache, use_cache=True,
                         logits_to_keep=1)
        return out.logits, cache

    @torch.no_grad()
    def prefill_e2e(self):
        """Public API from host memory: token ids H2D, the prefill, logits D2H."""
        ids = self.ids_host.to(self.dev, non_blocking=True)
        logits, cache = self.prefill(ids)
        self.logits_host.copy_(logits, non_blocking=True)
        return cache


def run_model(args, ws, rank, local, dev, peaks):
    hbm_peak, _tc_burst, tc_sus, peak_kind = peaks
    mb = ModelBench(dev, rank)
    # the swapped model with transformers' eager decoder-layer glue, for comparison
    mb.prefill()
    torch.cuda.synchronize()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(2):
        mb.prefill()
    e1.record()
    torch.cuda.synchronize()
    unfused_ms = _max_over_ranks(e0.elapsed_time(e1) / 2, ws)
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
    fuse_qwen_decoder_layers(mb.model)
    for _ in range(args.warmup):
        mb.prefill()
    torch.cuda.synchronize()
    sampler = ClockSampler(_gpu_index(local))
    sampler.start()
    _barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(args.steps):
        logits, cache = mb.prefill()
        del cache
    e1.record()
    torch.cuda.synchronize()
    _barrier(ws)
    clocks = sampler.stop()
    ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    value = MODEL_T * ws / (ms / 1000.0)

    # end to end through the public API from pinned host memory
    for _ in range(2):
        mb.prefill_e2e()
    torch.cuda.synchronize()
    e0.record()
    n_e2e = max(1, min(5, args.steps))
    for _ in range(n_e2e):
        mb.prefill_e2e()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / n_e2e, ws)

    # greedy decode (32 tokens) from a prefilled cache, captured in a CUDA graph
    decode = {"steps": MODEL_DECODE, "context": MODEL_T}
    try:
        logits, cache = mb.prefill()
        first = logits[:, -1].argmax(-1, keepdim=True)
        gd = mb.qt.GraphedGreedyDecode(mb.model, cache, first, MODEL_DECODE)
        for _ in range(3):
            gd.replay()
        torch.cuda.synchronize()
        same = bool(torch.equal(gd.tokens, gd.eager_tokens))
        reps = 10
        e0.record()
        for _ in range(reps):
            gd.replay()
        e1.record()
        torch.cuda.synchronize()
        us = _max_over_ranks(e0.elapsed_time(e1) * 1000.0 / (reps * MODEL_DECODE), ws)
        dbytes = model_decode_bytes_per_token(MODEL_T)
        dense = 2 * MODEL["kv_heads"] * MODEL["head_dim"] * 2 * (MODEL_T + MODEL_DECODE) * MODEL["layers"]
        decode.update({
            "us_per_token": round(us, 2), "tokens_per_s": round(1e6 / us * ws, 1),
            "graph_tokens_equal_eager": same,
            "algorithmic_bytes_per_token": dbytes, "achieved_gbs": round(dbytes / (us * 1e-6) / 1e9, 1),
            "hbm_frac": round(dbytes / (us * 1e-6) / 1e9 / hbm_peak, 4),
            "retained_kv_bytes": int(cache.nbytes), "dense_kv_bytes": int(dense),
            "path": "HF model forward per token (embedding, 24 swapped layers each one fused append+close+"
                    "attend launch, lm_head, argmax) for 32 tokens, recorded once in a CUDA graph and replayed"})
        del gd, cache
    except Exception as exc:  # noqa: BLE001 - report, keep the prefill number
        decode["error"] = f"{type(exc).__name__}: {exc}"[:400]
    torch.cuda.synchronize()

    # the attention kernel alone at this shape (HBM roofline beside the model's TC roofline)
    att = attention_kernel_at(dev, MODEL_T, MODEL["heads"], MODEL["kv_heads"], layer=MODEL["layers"] - 1,
                              reps=max(3, min(10, args.steps)), hbm_peak=hbm_peak)
    flops = model_prefill_flops(MODEL_T)
    achieved = flops / (ms / 1000.0) / 1e12  # per GPU: every rank runs one sequence of its own
    del mb
    torch.cuda.empty_cache()
    return {
        "value": value, "ms": ms, "clocks": clocks,
        "unfused": {"prefill_tok_per_s": round(MODEL_T * ws / (unfused_ms / 1000.0), 1), "ms_per_step": round(unfused_ms, 3),
                    "what": "same model and attention kernels with transformers' eager decoder-layer glue "
                            "(swap_qwen_attention_with_butterfly_cuda only, as the reference swaps)"},
        "e2e": {"value": round(MODEL_T * ws / (e2e_ms / 1000.0), 1), "unit": "tok/s",
                "h2d_bytes_per_step": MODEL_T * 8, "d2h_bytes_per_step": MODEL["vocab"] * 2,
                "path": "model(input_ids) from pinned host token ids (H2D inside the timed region), "
                        "next-token logits copied back to pinned host memory"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": tc_sus, "unit": "TFLOP/s",
                     "frac": round(achieved / tc_sus, 4), "traffic": None,
                     "peak_kind": f"{peak_kind} bf16_tflops_sustained (cuBLAS GEMM looped under the power cap)",
                     "flops_per_step": flops,
                     "flops_note": "2 x linear MACs per token (352.3M non-embedding params) + attention over "
                                   "selected keys + lm_head for the kept position; per GPU",
                     "traffic_note": "the step's dominant kernels are GEMMs (ours for q/k/v and gate/up, cuBLAS for o/down); DRAM traffic is given for "
                                     "the attention kernel below",
                     "attention_kernel": att},
        "decode": decode,
        "launches_per_step": 7 * MODEL["layers"] + 3,
    }


def attention_kernel_at(dev, seq_len, hq, hkv, layer, reps, hbm_peak):
    """CUDA-event time of the prefill kernel alone on seeded N(0,1) inputs of this shape."""
    import butterfly_b200 as bb
    from butterfly_b200.attention import block_mean_summaries_kv, prefill_attention_into, route_for
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(1, hq, seq_len, DH, device=dev, generator=g).bfloat16()
    k = torch.randn(1, hkv, seq_len, DH, device=dev, generator=g).bfloat16()
    v = torch.randn(1, hkv, seq_len, DH, device=dev, generator=g).bfloat16()
    lay = bb.build_block_butterfly_layout(seq_len=seq_len, block_size=BS, num_key_value_heads=hkv,
                                          num_key_value_groups=hq // hkv, layer_idx=layer, local_window_blocks=1,
                                          sink_count=1, partner_count=1, partner_rule="causal_shift")
    r = route_for(lay, dev)[0]
    N = lay.num_blocks
    ks, vs = block_mean_summaries_kv(k, v, seq_len=seq_len, block_size=BS, num_blocks=N)
    out = torch.empty(1, seq_len, hq, DH, device=dev, dtype=torch.bfloat16).transpose(1, 2)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    sc = 1.0 / math.sqrt(DH)
    for _ in range(3):
        prefill_attention_into(q, k, v, ks, vs, out, None, r, W, sc)
    ts, cs = [], []
    for _ in range(reps):
        flush.zero_()
        a, b, c = _events(3)
        a.record()
        block_mean_summaries_kv(k, v, seq_len=seq_len, block_size=BS, num_blocks=N, k_out=ks, v_out=vs)
        b.record()
        prefill_attention_into(q, k, v, ks, vs, out, None, r, W, sc)
        c.record()
        torch.cuda.synchronize()
        cs.append(a.elapsed_time(b))
        ts.append(b.elapsed_time(c))
    ms = sum(ts) / len(ts)
    cms = sum(cs) / len(cs)
    byts = prefill_bytes_per_launch(seq_len, hq, hkv)
    cb = compress_bytes_per_pair(seq_len, hkv)
    return {"kernel": "prefill_sm100_kernel", "seq_len": seq_len, "bound": "hbm", "bytes_per_launch": byts,
            "ms_per_launch": round(ms, 5), "achieved": round(byts / (ms / 1000) / 1e9, 1), "peak": hbm_peak,
            "unit": "GB/s", "frac": round(byts / (ms / 1000) / 1e9 / hbm_peak, 4),
            "traffic": _traffic_from_profiles("prefill_128k"),
            "compressor_pair_ms": round(cms, 5),
            "compressor_gbs": round(cb / (cms / 1000) / 1e9, 1), "l2": "flushed (2x L2 write) before each launch"}


# ----------------------------------------------------------------------------- sequence shard (262k)
SHARD_MODEL = dict(hidden=2560, layers=32, heads=16, kv_heads=4, head_dim=128, inter=9728, vocab=151936)
SHARD_T = 262144


def retained_kv_bytes(total: int, spec, chunk: int = MODEL_CHUNK, decode_tokens: int = 0) -> int:
    """Bytes a two-pool cache keeps for a ``total``-token prompt handed over in ``chunk``
    chunks, then ``decode_tokens`` one-token steps (tail rows + closed block means, K and V,
    bf16, every layer): the same counter arithmetic the cache runs."""
    from butterfly_b200.cache import CompressedKVCache
    c = CompressedKVCache(block_size=BS, local_window_tokens=W, max_kv_size=total + 64, max_chunk_size=chunk)
    c.tail_capacity = W + 2 * chunk + 2 * BS
    c.summary_capacity = (total + 64) // BS + 4
    c._advance_counters_chunked(total, chunk)
    for _ in range(decode_tokens):
        c._advance_counters_chunked(1, 1)
    return 2 * spec["kv_heads"] * spec["head_dim"] * 2 * (c.tail_size + c.summary_count) * spec["layers"]


def run_seq_shard(args, ws, rank, dev, peaks):
    """The 4B-class model's 262144-token prefill, sequence-sharded over the ranks (strong
    scaling: one sequence, T / n_gpus tokens per GPU; NCCL all-gathers of block means and
    the W-1-token halo in every layer)."""
    from butterfly_b200.integrations import qwen_torch as qt
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
    tc_sus = peaks[2]
    if SHARD_T % (ws * BS):
        return {"error": f"T={SHARD_T} does not split into whole blocks over {ws} ranks"}
    model = build_model(dev, seed=2, spec=SHARD_MODEL)
    fuse_qwen_decoder_layers(model)
    Tl = SHARD_T // ws
    g = torch.Generator().manual_seed(2000)
    ids = torch.randint(0, SHARD_MODEL["vocab"], (1, SHARD_T), generator=g)[:, rank * Tl:(rank + 1) * Tl].to(dev)
    pos = torch.arange(rank * Tl, (rank + 1) * Tl, device=dev).view(1, -1)

    @torch.no_grad()
    def step():
        with qt.sequence_sharded(model, SHARD_T):
            return model(input_ids=ids, position_ids=pos, use_cache=False, logits_to_keep=1).logits

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    n = max(1, min(3, args.steps))
    _barrier(ws)
    e0, e1 = _events(2)
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / n, ws)
    flops = model_linear_flops_per_token(SHARD_MODEL) * SHARD_T + sum(
        4 * SHARD_MODEL["head_dim"] * SHARD_MODEL["heads"] * attention_valid_keys(SHARD_T, l)
        for l in range(SHARD_MODEL["layers"])) + 2 * SHARD_MODEL["hidden"] * SHARD_MODEL["vocab"]
    tflops = flops / (ms / 1000.0) / 1e12
    per_layer_exchange = 2 * SHARD_MODEL["kv_heads"] * (SHARD_T // BS) * SHARD_MODEL["head_dim"] * 2
    out = {"workload": f"4B-class Qwen3.5 decoder (seed 2): 32 layers, hidden 2560, Hq16/Hkv4, dh128, SwiGLU 9728, "
                       f"vocab 151936, compressed Butterfly BS128 W64 + fused glue; one {SHARD_T}-token prefill "
                       f"sequence-sharded over {ws} GPU(s) ({Tl} tokens each), use_cache=False, logits_to_keep=1",
           "scaling": "strong", "prefill_tok_per_s": round(SHARD_T / (ms / 1000.0), 1), "ms_per_step": round(ms, 2),
           "steps": n, "tensor_roofline": {"achieved": round(tflops, 1), "peak": round(tc_sus * ws, 1),
                                           "frac": round(tflops / (tc_sus * ws), 4), "unit": "TFLOP/s",
                                           "note": "whole-job FLOPs over the measured sustained bf16 peak x n_gpus"},
           "all_gather_bytes_per_layer": per_layer_exchange + ws * 2 * (W - 1) * SHARD_MODEL["kv_heads"] * 128 * 2,
           "retained_kv_bytes_after_prefill": retained_kv_bytes(SHARD_T, SHARD_MODEL),
           "retained_kv_bytes_after_one_decode_token": retained_kv_bytes(SHARD_T, SHARD_MODEL, decode_tokens=1),
           "retained_kv_note": "two-pool cache counters for the prompt handed over in 4096-token chunks "
                               "(kv_step of the reference harness); the tail trims to the window at the first "
                               "decode token",
           "dense_kv_bytes": 2 * SHARD_MODEL["kv_heads"] * SHARD_MODEL["head_dim"] * 2 * SHARD_T * SHARD_MODEL["layers"]}
    del model
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- layer (32k)
def _layouts(seq_len):
    import butterfly_b200 as bb
    return [bb.build_block_butterfly_layout(seq_len=seq_len, block_size=BS, num_key_value_heads=HKV,
                                            num_key_value_groups=HQ // HKV, layer_idx=l, local_window_blocks=1,
                                            sink_count=1, partner_count=1, partner_rule="causal_shift")
            for l in LAYERS]


def prefill_bytes_per_launch(seq_len=T, hq=HQ, hkv=HKV) -> int:
    """Algorithmic HBM bytes of one prefill-kernel launch: read Q, K, V and the routed block
    means, write O (bf16).  Summaries are read once per (block, KV head)."""
    N = -(-seq_len // BS)
    return 2 * DH * seq_len * (hq + 2 * hkv + hq) + 2 * 2 * hkv * N * DH


def compress_bytes_per_pair(seq_len=T, hkv=HKV) -> int:
    N = -(-seq_len // BS)
    return 2 * (2 * DH * seq_len * hkv) + 2 * (2 * DH * N * hkv)


def run_prefill(dev, seed, steps, warmup):
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
    ev = [[_events(3) for _ in LAYERS] for _ in range(steps)]

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


def run_layer(args, ws, dev, hbm_peak, rank):
    """One attention layer at T=32768, stages 0..7 per step (CUDA-graph replay)."""
    step, ev, ins, lays = run_prefill(dev, 1000 + rank, args.steps, args.warmup)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step()
    for _ in range(args.warmup):
        graph.replay()
    _barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    # per-kernel durations: the same steps launched eagerly, each kernel bracketed by events
    # on its stream.  A device-side sleep queued first lets the host enqueue the whole pass
    # before the GPU reaches it, so no launch waits on the host.
    torch.cuda._sleep(int(2e8))
    for si in range(args.steps):
        step(si)
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    pf = [ev[s][i][1].elapsed_time(ev[s][i][2]) for s in range(args.steps) for i in range(len(LAYERS))]
    cp = [ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps) for i in range(len(LAYERS))]
    pf_ms, cp_ms = sum(pf) / len(pf), sum(cp) / len(cp)
    e2e_ms, h2d, d2h = run_layer_e2e(dev, lays, ins, max(1, min(3, args.steps)))
    e2e_ms = _max_over_ranks(e2e_ms, ws)
    del ins
    torch.cuda.empty_cache()
    pf_bytes = prefill_bytes_per_launch()
    achieved = pf_bytes / (pf_ms / 1000.0) / 1e9
    return {
        "workload": "one compressed-attention layer, T=32768, Hq8/Hkv2, dh128, BS128, W64, causal_shift layers "
                    "0-7 (stages 0-7, partner offsets 1..128) per step, seeded N(0,1) Q/K/V per layer "
                    f"({len(LAYERS) * 2 * DH * T * (HQ + 2 * HKV) / 2**20:.0f} MiB per step > L2); "
                    "compressor + tcgen05 prefill, CUDA-graph replay",
        "layer_tok_per_s": round(len(LAYERS) * T * ws / (ms / 1000.0), 1), "ms_per_step": round(ms, 4),
        "e2e_layer_tok_per_s": round(len(LAYERS) * T * ws / (e2e_ms / 1000.0), 1),
        "e2e_h2d_bytes_per_step": h2d, "e2e_d2h_bytes_per_step": d2h,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": _traffic_from_profiles("prefill_c2"),
                     "kernel": "prefill_sm100_kernel", "bytes_per_launch": pf_bytes,
                     "ms_per_launch": round(pf_ms, 5), "compressor_pair_ms": round(cp_ms, 5),
                     "compressor_gbs": round(compress_bytes_per_pair() / (cp_ms / 1000.0) / 1e9, 1)},
        "launches_per_step": 2 * len(LAYERS),
    }


def run_layer_e2e(dev, lays, ins, steps):
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
    e0, e1 = _events(2)
    e0.record()
    run(steps)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, h2d, d2h


# ----------------------------------------------------------------------------- batched decode
DEC_B, DEC_CTX, DEC_STEPS, DEC_CHUNK = 64, 65536, 128, 4096


def decode_bytes_per_step() -> int:
    """Per step, per (sequence, KV head): raw window K+V (W rows), <=2 routed summaries (K+V),
    the query heads and outputs, the appended token (read + ring write) and the amortised
    block close (BS rows of K and V read once every BS steps, plus the summary writes)."""
    row = DH * 2
    g = HQ // HKV
    per = 2 * W * row + 2 * 2 * row + 2 * g * row + 2 * 2 * row + (2 * BS * row + 2 * row) / BS
    return int(per * DEC_B * HKV)


def decode_inputs(dev, seed, B=DEC_B, ctx=DEC_CTX, steps=DEC_STEPS, keep=0):
    """The batched-decode workload: a two-pool cache holding B sequences of ``ctx`` seeded
    N(0,1) tokens (appended in chunks of DEC_CHUNK) and per-step q / k / v.  With ``keep``
    > 0 the first ``keep`` sequences of every input are also returned on the host."""
    from butterfly_b200.cache import CompressedKVCache
    g = torch.Generator(device=dev).manual_seed(seed)
    cache = CompressedKVCache(block_size=BS, local_window_tokens=W, max_kv_size=ctx + steps,
                              max_chunk_size=DEC_CHUNK)
    host_chunks = []
    for c0 in range(0, ctx, DEC_CHUNK):
        k = torch.randn(B, HKV, DEC_CHUNK, DH, device=dev, generator=g).bfloat16()
        v = torch.randn(B, HKV, DEC_CHUNK, DH, device=dev, generator=g).bfloat16()
        cache.append(k, v)
        if keep:
            host_chunks.append((k[:keep].cpu(), v[:keep].cpu()))
    q = torch.randn(steps, B, HQ, 1, DH, device=dev, generator=g).bfloat16()
    kn = torch.randn(steps, B, HKV, 1, DH, device=dev, generator=g).bfloat16()
    vn = torch.randn(steps, B, HKV, 1, DH, device=dev, generator=g).bfloat16()
    return cache, q, kn, vn, host_chunks


def decode_layouts(ctx=DEC_CTX, steps=DEC_STEPS, layer=3):
    import butterfly_b200 as bb
    return [bb.build_block_butterfly_layout(seq_len=ctx + s + 1, block_size=BS, num_key_value_heads=HKV,
                                            num_key_value_groups=HQ // HKV, layer_idx=layer, local_window_blocks=1,
                                            sink_count=1, partner_count=1, partner_rule="causal_shift")
            for s in range(steps)]


def run_decode(dev, seed, reps, warmup):
    cache, q, kn, vn, _ = decode_inputs(dev, seed)
    lays = decode_layouts()
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
    e0, e1 = _events(2)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * DEC_STEPS)
    return us, cache


def launch_floor_us(dev, ctas: int, n: int = 128) -> float:
    """Per-launch time of a graph of ``n`` empty dependent launches (programmatic dependent
    launch, ``ctas`` CTAs each): the floor under a chain of decode steps."""
    from butterfly_b200 import _lib
    s = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        for _ in range(3):
            _lib.check(_lib.lib().bna_launch_probe(ctas, _lib.stream_ptr(dev)))
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            for _ in range(n):
                _lib.check(_lib.lib().bna_launch_probe(ctas, _lib.stream_ptr(dev)))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(10):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / (10 * n)


def run_batched_decode(ws, dev, hbm_peak, rank):
    us, cache = run_decode(dev, 2000 + rank, reps=10, warmup=3)
    us = _max_over_ranks(us, ws)
    gbs = decode_bytes_per_step() / (us * 1e-6) / 1e9
    out = {"workload": "B=64 sequences x 65536 pre-filled tokens (two-pool cache, chunks of 4096), Hq8/Hkv2, dh128, "
                       "BS128, W64; 128 fused append+close+attend steps, CUDA-graph replay",
           "us_per_step": round(us, 3), "sequences_per_step": DEC_B * ws,
           "algorithmic_bytes_per_step": decode_bytes_per_step(),
           "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 4),
           "launch_floor_us": round(launch_floor_us(dev, DEC_B * HKV), 3),
           "launch_floor_note": "graph of 128 empty dependent launches of 128 CTAs (bna_launch_probe)",
           "retained_kv_bytes_per_layer": cache.nbytes,
           "dense_kv_bytes_per_layer": 2 * DEC_B * HKV * (DEC_CTX + DEC_STEPS) * DH * 2}
    del cache
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- CPU legs
def cpu_port_layer_seconds(layer: int, seed: int = 0) -> float:
    """One 32k attention-layer pass of the reference's CPU algorithm (oracle/torch_port.py, fp32)."""
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


class CPUModelLayer:
    """One decoder layer of the model workload in fp32 on the host, with its attention
    computed by the reference's algorithm (oracle/torch_port.py: gather + masked SDPA),
    as the reference's swapped module does on CPU (qwen_torch.py:1461-1470, 1585-1591)."""

    def __init__(self, layer_idx: int, seed: int = 1):
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5DecoderLayer, Qwen3_5TextRotaryEmbedding
        cfg = model_config()
        torch.manual_seed(seed)
        self.layer = Qwen3_5DecoderLayer(cfg, layer_idx).eval()
        for mod in self.layer.modules():
            if isinstance(mod, torch.nn.Linear):
                torch.nn.init.normal_(mod.weight, std=0.02)
        self.rotary = Qwen3_5TextRotaryEmbedding(cfg)
        self.layer_idx = layer_idx

    @torch.no_grad()
    def forward(self, x: torch.Tensor, positions: torch.Tensor, kv=None):
        from butterfly_b200.integrations.qwen_torch import extract_qkv_from_qwen_attention
        from oracle import topology as ot
        from oracle import torch_port
        L = self.layer
        attn = L.self_attn
        pe = self.rotary(x, positions.view(1, -1))
        h = L.input_layernorm(x)
        q, k, v, gate = extract_qkv_from_qwen_attention(attn, h, pe)
        n_tok = int(x.shape[1])
        if kv is None:  # prefill
            nb = ot.block_neighbors_table(-(-n_tok // BS), self.layer_idx, local_window_blocks=1, sink_count=1,
                                          partner_count=1, partner_rule="causal_shift")
            y = torch_port.prefill(q, k, v, nb, block_size=BS, window=W)
        else:  # one decode token over the full history (the reference recomputes every summary)
            kk, vv = torch.cat([kv[0], k], 2), torch.cat([kv[1], v], 2)
            tk = int(kk.shape[2])
            nb = ot.block_neighbors_table(-(-tk // BS), self.layer_idx, local_window_blocks=1, sink_count=1,
                                          partner_count=1, partner_rule="causal_shift")
            y = torch_port.active(q, kk, vv, nb, [tk - 1], block_size=BS, window=W)
        y = y.transpose(1, 2).reshape(1, n_tok, -1) * torch.sigmoid(gate)
        x = x + attn.o_proj(y)
        return x + L.mlp(L.post_attention_layernorm(x))


CPU_SAMPLE_T = 16384  # host sample length of one decoder layer; per-token cost is constant in T


def cpu_model_layer_seconds(lay: "CPUModelLayer", seq_len: int, seed: int = 0) -> float:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, seq_len, MODEL["hidden"], generator=g)
    t0 = time.perf_counter()
    lay.forward(x, torch.arange(seq_len))
    return time.perf_counter() - t0


def cpu_model_decode_layer_seconds(lay: "CPUModelLayer", ctx: int, seed: int = 0) -> float:
    """One decode token of one layer over a ``ctx``-token history (reference algorithm)."""
    g = torch.Generator().manual_seed(seed)
    kv = (torch.randn(1, HKV, ctx, DH, generator=g), torch.randn(1, HKV, ctx, DH, generator=g))
    x = torch.randn(1, 1, MODEL["hidden"], generator=g)
    t0 = time.perf_counter()
    lay.forward(x, torch.tensor([ctx]), kv)
    return time.perf_counter() - t0


def cpu_lm_head_seconds() -> float:
    w = torch.randn(MODEL["vocab"], MODEL["hidden"]) * 0.02
    x = torch.randn(1, MODEL["hidden"])
    (x @ w.t()).argmax(-1)
    t0 = time.perf_counter()
    for _ in range(5):
        (x @ w.t()).argmax(-1)
    return (time.perf_counter() - t0) / 5


CPU_DEC_B = 8  # host sample of the batched decode: 8 of the 64 sequences (cost is linear in B)


def cpu_batched_decode_seconds(steps: int = 2) -> float:
    """Reference decode (all summaries recomputed over the full history) at the batched-decode
    shapes with CPU_DEC_B sequences, 65536+1 keys, one query token per sequence; median over
    ``steps`` steps, scaled to the 64 sequences of the workload."""
    from oracle import topology as ot
    from oracle import torch_port
    g = torch.Generator().manual_seed(5)
    k = torch.randn(CPU_DEC_B, HKV, DEC_CTX + 1, DH, generator=g)
    v = torch.randn(CPU_DEC_B, HKV, DEC_CTX + 1, DH, generator=g)
    nb = ot.block_neighbors_table(-(-(DEC_CTX + 1) // BS), 3, local_window_blocks=1, sink_count=1,
                                  partner_count=1, partner_rule="causal_shift")
    ts = []
    for s in range(steps + 1):
        q = torch.randn(CPU_DEC_B, HQ, 1, DH, generator=g)
        t0 = time.perf_counter()
        torch_port.active(q, k, v, nb, [DEC_CTX], block_size=BS, window=W)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts[1:]) * DEC_B / CPU_DEC_B


def cpu_baseline(n_samples: int = 3):
    torch.set_num_threads(os.cpu_count() or 1)
    Ls = MODEL["layers"]
    lay = CPUModelLayer(Ls - 1)
    cpu_model_layer_seconds(lay, CPU_SAMPLE_T)  # warm-up (first-touch of the activations)
    t_layer = statistics.median([cpu_model_layer_seconds(lay, CPU_SAMPLE_T, seed=i) for i in range(n_samples)])
    cpu_model_decode_layer_seconds(lay, MODEL_T)
    t_dec_layer = cpu_model_decode_layer_seconds(lay, MODEL_T, seed=1)
    t_head = cpu_lm_head_seconds()
    t_bdec = cpu_batched_decode_seconds()
    scale = MODEL_T / CPU_SAMPLE_T
    prefill_s = Ls * t_layer * scale
    decode_s = Ls * t_dec_layer + t_head
    return {"value": round(MODEL_T / prefill_s, 1), "unit": "tok/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"one decoder layer of the model workload in fp32 with the reference's attention algorithm "
                      f"(oracle/torch_port.py: gather + masked SDPA) on a {CPU_SAMPLE_T}-token prompt, median of "
                      f"{n_samples} ({t_layer:.3f} s); the {MODEL_T}-token model prefill = {Ls} layers x "
                      f"{scale:.0f} x that (every term of the layer is linear in T)",
            "decode_us_per_token": round(decode_s * 1e6, 1),
            "decode_sample": f"one decode token of one layer over a {MODEL_T}-token history ({t_dec_layer:.3f} s; "
                             f"the reference recomputes every block summary each step) x {Ls} + lm_head "
                             f"({t_head * 1000:.1f} ms)",
            "batched_decode_us_per_step": round(t_bdec * 1e6, 1),
            "batched_decode_sample": f"median of 2 reference decode steps (after one warm-up) at B={CPU_DEC_B}, 65537 keys, "
                                     f"Hq8/Hkv2 (fp32), x{DEC_B // CPU_DEC_B} for the 64 sequences"}


# ----------------------------------------------------------------------------- reference arm
def reference_gpu(dev):
    """The reference's algorithm (gather + boolean-mask SDPA, oracle/torch_port.py) run by
    torch on the B200 in bf16: the model workload's prefill with that attention in every
    layer, and one 32k attention layer (the reference's engine="sdpa" route)."""
    from oracle import topology as ot
    from oracle import torch_port

    from butterfly_b200.integrations import qwen_torch as qt

    class _RefAttention:
        @staticmethod
        def butterfly_compressed_attention(q, k, v, *, layout, local_window_tokens, **_):
            return torch_port.prefill(q, k, v, layout.block_neighbors[0].tolist(), block_size=layout.block_size,
                                      window=local_window_tokens)

    res = {}
    g = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn(1, HQ, T, DH, device=dev, generator=g).bfloat16()
    k = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
    v = torch.randn(1, HKV, T, DH, device=dev, generator=g).bfloat16()
    nb = ot.block_neighbors_table(T // BS, 5, local_window_blocks=1, sink_count=1, partner_count=1,
                                  partner_rule="causal_shift")
    for _ in range(2):
        torch_port.prefill(q, k, v, nb, block_size=BS, window=W)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        torch_port.prefill(q, k, v, nb, block_size=BS, window=W)
    torch.cuda.synchronize()
    res["layer_tok_per_s"] = round(T * 5 / (time.perf_counter() - t0), 1)
    del q, k, v
    saved = qt._attn
    qt._attn = _RefAttention
    try:
        mb = ModelBench(dev, 0)
        with torch.no_grad():
            mb.model(input_ids=mb.ids, use_cache=False, logits_to_keep=1)
            torch.cuda.synchronize()
            ts = []
            for _ in range(2):
                t0 = time.perf_counter()
                mb.model(input_ids=mb.ids, use_cache=False, logits_to_keep=1)
                torch.cuda.synchronize()
                ts.append(time.perf_counter() - t0)
        res["model_prefill_tok_per_s"] = round(MODEL_T / min(ts), 1)
        del mb
    except Exception as exc:  # noqa: BLE001
        res["model_error"] = f"{type(exc).__name__}: {exc}"[:300]
    finally:
        qt._attn = saved
    torch.cuda.empty_cache()
    res["note"] = ("reference algorithm restated in oracle/torch_port.py (index tables built on the host, "
                   "gather + masked SDPA on the GPU), bf16, host-timed with cuda synchronize")
    return res


def run_reference(args, ws, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    Ls = MODEL["layers"]
    Ts = CPU_SAMPLE_T
    lay = CPUModelLayer(Ls - 1)
    for i in range(args.warmup):
        cpu_model_layer_seconds(lay, Ts, seed=i)
    times = [cpu_model_layer_seconds(lay, Ts, seed=100 + i) for i in range(args.steps)]
    per_layer = sum(times) / len(times)
    per = per_layer * Ls * (MODEL_T / Ts)
    val = MODEL_T / per
    ref_gpu = None
    if torch.cuda.is_available():
        try:
            ref_gpu = reference_gpu(torch.device("cuda", 0))
        except Exception as exc:  # noqa: BLE001
            ref_gpu = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    line = {
        "impl": "reference", "metric": "prefill_tok_per_s", "value": round(val, 1), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded random-init weights and uniform random token ids / N(0,1) activations",
        "config": {"workload": f"model-128k: 0.8B-class Qwen3.5 decoder (24 layers, hidden 1024, Hq8/Hkv2, dh128, "
                               f"SwiGLU 3584, vocab 151936), compressed Butterfly attention BS128 W64, prefill "
                               f"T={MODEL_T}; each step times one decoder layer on a {Ts}-token prompt on the host; "
                               f"model time = {Ls} layers x {MODEL_T // Ts} x that (bounded CPU sample)",
                   "seq_len": MODEL_T},
        "cpu_baseline": {"value": round(val, 1), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"one {Ts}-token decoder layer per step (fp32, attention by "
                                   f"oracle/torch_port.py), x{Ls} layers x {MODEL_T // Ts}"},
        "e2e": {"value": round(val, 1), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu": ref_gpu,
    }
    print(json.dumps(line), flush=True)


def _traffic_from_profiles(name: str):
    p = os.path.join(ROOT, "profiles", f"{name}_ncu.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


# ----------------------------------------------------------------------------- profiling cases
def prefill_trace(dev):
    """Per-unit pipeline timeline of one 32k prefill launch (globaltimer stamps)."""
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
    """Small, self-terminating cases for ncu captures (a few hundred MB on the device)."""
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
    elif kind == "prefill-128k":
        # the model workload's attention shape (T=131072, Hq8/Hkv2): warm-up, then one launch
        att = attention_kernel_at(dev, MODEL_T, MODEL["heads"], MODEL["kv_heads"], layer=MODEL["layers"] - 1, reps=1,
                                  hbm_peak=_peaks()[0])
        print(att)
    elif kind == "model-decode":
        # greedy decode tokens of the fused model after a 128k prefill, inside an NVTX range
        # named "decode" (ncu --nvtx --nvtx-include decode/)
        from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
        mb = ModelBench(dev, 0)
        fuse_qwen_decoder_layers(mb.model)
        with torch.no_grad():
            logits, cache = mb.prefill()
            tok = logits[:, -1].argmax(-1, keepdim=True)
            for i in range(4):
                if i == 2:
                    torch.cuda.synchronize()
                    torch.cuda.nvtx.range_push("decode")
                out = mb.model(input_ids=tok, past_key_values=cache, use_cache=True)
                tok = out.logits[:, -1].argmax(-1, keepdim=True)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    elif kind == "model-prefill":
        from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
        mb = ModelBench(dev, 0)
        fuse_qwen_decoder_layers(mb.model)
        mb.prefill()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("prefill")
        mb.prefill()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    elif kind == "gemm-down":
        # the model's down projection onto the residual (in place, with the next norm's row
        # statistics) at T=131072: 3 warm-up launches, then one
        from butterfly_b200 import glue
        g = torch.Generator(device=dev).manual_seed(0)
        H, I = MODEL["hidden"], MODEL["inter"]
        act = torch.randn(MODEL_T, I, device=dev, generator=g).bfloat16()
        wd = (torch.randn(H, I, device=dev, generator=g) / I ** 0.5).bfloat16()
        x2 = torch.randn(MODEL_T, H, device=dev, generator=g).bfloat16()
        ss = torch.empty(MODEL_T, 4 * (H // 256), device=dev, dtype=torch.float32)
        for _ in range(4):
            glue.gemm_residual(act, wd, x2, out=x2, ss_out=ss)
    elif kind in ("gemm-swiglu", "gemm-qkv"):
        # the model's gate/up (or q/k/v) projection at T=131072: 3 warm-up launches, then one
        from butterfly_b200 import glue
        g = torch.Generator(device=dev).manual_seed(0)
        H = MODEL["hidden"]
        h = torch.randn(1, MODEL_T, H, device=dev, generator=g).bfloat16()
        if kind == "gemm-swiglu":
            w = (torch.randn(2 * MODEL["inter"], H, device=dev, generator=g) / H ** 0.5).bfloat16()
            fn = lambda: glue.gemm_swiglu(h, w, MODEL["inter"])  # noqa: E731
        else:
            hq, hkv, dh = MODEL["heads"], MODEL["kv_heads"], MODEL["head_dim"]
            w = (torch.randn((2 * hq + 2 * hkv) * dh, H, device=dev, generator=g) / H ** 0.5).bfloat16()
            nw = torch.ones(dh, device=dev, dtype=torch.bfloat16)
            cs = torch.randn(1, MODEL_T, 32, device=dev, generator=g).bfloat16()
            fn = lambda: glue.gemm_qkv_norm_rope(h, w, hq, hkv, nw, nw, cs, cs, 1e-6)  # noqa: E731
        for _ in range(4):
            fn()
    else:
        run_decode(dev, 0, reps=1, warmup=1)
    torch.cuda.synchronize()
    print("profile case done", flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-layer", action="store_true", help="skip the 32k attention-layer leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the batched-decode leg")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-shard", action="store_true", help="skip the sequence-sharded 262k leg")
    ap.add_argument("--profile-case", choices=["prefill", "decode", "prefill-trace", "model-prefill", "model-decode", "prefill-128k", "gemm-down",
                                                      "gemm-swiglu", "gemm-qkv"], default=None,
                    help="small case for ncu: warm-up, then the launches to capture")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    ws, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = _peaks()
    hbm_peak = peaks[0]

    m = run_model(args, ws, rank, local, dev, peaks)
    shard = None if args.no_shard else run_seq_shard(args, ws, rank, dev, peaks)
    layer = None if args.no_layer else run_layer(args, ws, dev, hbm_peak, rank)
    bdec = None if args.no_decode else run_batched_decode(ws, dev, hbm_peak, rank)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_baseline()

    line = {
        "metric": "prefill_tok_per_s", "value": round(m["value"], 1), "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(m["ms"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init weights (seed 1), uniform random token ids (seeded per rank)",
        "config": {"workload": f"model-128k: 0.8B-class Qwen3.5 decoder, 24 layers, hidden 1024, Hq8/Hkv2, dh128, "
                               f"SwiGLU 3584, vocab 151936, every layer compressed Butterfly attention (BS128, W64, "
                               f"causal_shift) plus fused decoder-layer glue (fuse_qwen_decoder_layers); prefill "
                               f"T={MODEL_T} into a fresh two-pool cache, logits_to_keep=1; "
                               f"then {MODEL_DECODE} greedy decode steps",
                   "global_batch": ws, "seq_len": MODEL_T, "parallelism": f"batch-sharded x{ws} (one sequence per GPU)",
                   "l2": "inputs larger than L2: 1.33 GB of weights and >=0.27 GB activations per layer pass"},
        "roofline": m["roofline"],
        "cpu_baseline": cpu,
        "e2e": m["e2e"],
        "gpu_launches": args.steps * m["launches_per_step"],
        "gpu_launches_note": "our kernels per prefill: per layer the q/k/v GEMM (input RMSNorm folded in, q/k "
                             "norm+RoPE epilogue), compressor, gated prefill kernel, cache hand-off append, o_proj "
                             "GEMM + residual, gate/up GEMM (post-attention RMSNorm folded in, SwiGLU epilogue), "
                             "down GEMM + residual (7); plus the first layer's row statistics, the final norm and "
                             "the lm_head GEMV; no cuBLAS kernel runs in the prefill (ncu launch list)",
        "timing": "CUDA events around the timed prefills; decode from CUDA-graph replays",
        "clocks": m["clocks"],
        "decode": m["decode"],
        "prefill_unfused_glue": m["unfused"],
        "seq_shard": shard,
        "layer": layer,
        "decode_batched": bdec,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
