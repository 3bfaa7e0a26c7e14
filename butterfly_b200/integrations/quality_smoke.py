"""Quality smoke: compressed Butterfly against stock attention on the same Qwen3.5 model.

Product-level check of the reference's ``scripts/quality_smoke.py`` (there on MLX):
the model runs prefill on a deterministic prompt and greedy-decodes a short suffix once
with stock (dense) attention and once swapped onto the B200 compressed kernels, then

* KL of the next-token distributions at the end of prefill, both directions, over the
  stock top-k tokens that also appear in the compressed top-k (reference ``_kl``, :228-238)
* top-k overlap and top-1 agreement of those distributions (:241-262)
* exact match and token-by-token agreement of the greedy suffix.

The smoke is descriptive, as the reference's: it reports, it does not assert.

    python -m butterfly_b200.integrations.quality_smoke --seq-len 8192 --decode-len 32 \\
        [--model-path /path/to/qwen3.5]       # random-init 0.8B-class model without it
"""
from __future__ import annotations

import argparse
import json
import math
from typing import Any, Dict, List

import torch


def run_mode(model, input_ids: torch.Tensor, decode_len: int, top_k: int = 50, cache=None) -> Dict[str, Any]:
    """Prefill ``input_ids`` [1, T] and greedy-decode ``decode_len`` tokens.  Returns the
    final prefill distribution's top-k (token id, logit, log-prob) and the decoded ids."""
    with torch.no_grad():
        out = model(input_ids=input_ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        logits = out.logits[0, -1].float()
        logp = torch.log_softmax(logits, -1)
        top = torch.topk(logits, top_k)
        cache = out.past_key_values
        tok = top.indices[:1].view(1, 1)
        decoded: List[int] = [int(tok)]
        for _ in range(decode_len - 1):
            out = model(input_ids=tok, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            decoded.append(int(tok))
    return {"final_log_softmax_top_k": [{"token_id": int(i), "logit": float(l), "log_prob": float(logp[i])}
                                        for i, l in zip(top.indices.tolist(), top.values.tolist())],
            "decoded_ids": decoded}


def kl_over_overlap(p_log: Dict[int, float], q_log: Dict[int, float]) -> float:
    """KL(p || q) over the tokens of p that q also lists (nan without overlap)."""
    kl, overlap = 0.0, 0
    for tok, lp in p_log.items():
        if tok in q_log:
            kl += math.exp(lp) * (lp - q_log[tok])
            overlap += 1
    return kl if overlap > 0 else float("nan")


def compare(stock: Dict[str, Any], compressed: Dict[str, Any]) -> Dict[str, Any]:
    p = {e["token_id"]: e["log_prob"] for e in stock["final_log_softmax_top_k"]}
    q = {e["token_id"]: e["log_prob"] for e in compressed["final_log_softmax_top_k"]}
    a, b = stock["decoded_ids"], compressed["decoded_ids"]
    n = min(len(a), len(b))
    return {
        "top_k_overlap": len(set(p) & set(q)),
        "top_k_total": len(p),
        "kl_stock_compressed": kl_over_overlap(p, q),
        "kl_compressed_stock": kl_over_overlap(q, p),
        "top1_agree": stock["final_log_softmax_top_k"][0]["token_id"] == compressed["final_log_softmax_top_k"][0]["token_id"],
        "greedy_exact_match": a == b,
        "greedy_token_agreement": (sum(int(x == y) for x, y in zip(a, b)) / n) if n else float("nan"),
    }


def prompt_ids(vocab: int, seq_len: int, seed: int = 42) -> torch.Tensor:
    """Deterministic structured prompt: a fixed random passage of 512 ids repeated to length
    (the reference repeats a text passage; repetition gives attention a strong signal)."""
    g = torch.Generator().manual_seed(seed)
    base = torch.randint(0, vocab, (512,), generator=g)
    reps = -(-seq_len // 512)
    return base.repeat(reps)[:seq_len].view(1, -1)


def quality_smoke(model, input_ids: torch.Tensor, decode_len: int = 32, top_k: int = 50,
                  fused: bool = True) -> Dict[str, Any]:
    """Run ``model`` (stock Qwen3.5 attention) both ways and compare; the model is left
    with its stock attention restored."""
    from transformers import DynamicCache

    from . import qwen_torch as qt
    from .qwen_fused import fuse_qwen_decoder_layers, unfuse_qwen_decoder_layers
    qt.patch_qwen35_full_attention_decode()
    stock = run_mode(model, input_ids, decode_len, top_k, DynamicCache(config=model.config))
    qt.swap_qwen_attention_with_butterfly_cuda(model, qt.compressed_config())
    if fused:
        fuse_qwen_decoder_layers(model)
    try:
        cache = qt.make_compressed_cache(model, DynamicCache(config=model.config),
                                         max_kv_size=int(input_ids.shape[1]) + decode_len + 64,
                                         max_chunk_size=4096)
        comp = run_mode(model, input_ids, decode_len, top_k, cache)
    finally:
        unfuse_qwen_decoder_layers(model)
        qt.restore_qwen_dense_attention(model)
    return {"metrics": compare(stock, comp), "stock": stock, "compressed": comp,
            "seq_len": int(input_ids.shape[1]), "decode_len": decode_len}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model-path", default=None, help="local Qwen3.5 checkpoint; random-init 0.8B-class without")
    ap.add_argument("--seq-len", type=int, default=8192)
    ap.add_argument("--decode-len", type=int, default=32)
    ap.add_argument("--top-k", type=int, default=50)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--out-path", default=None)
    args = ap.parse_args()
    dev = torch.device("cuda")
    if args.model_path:
        from transformers import AutoModelForCausalLM
        model = AutoModelForCausalLM.from_pretrained(args.model_path, dtype=torch.bfloat16).to(dev).eval()
    else:
        from transformers import Qwen3_5TextConfig
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM
        cfg = Qwen3_5TextConfig(hidden_size=1024, intermediate_size=3584, num_hidden_layers=24, num_attention_heads=8,
                                num_key_value_heads=2, head_dim=128, vocab_size=151936,
                                layer_types=["full_attention"] * 24, max_position_embeddings=262144)
        torch.manual_seed(args.seed)
        with torch.device(dev):
            model = Qwen3_5ForCausalLM(cfg)
        model = model.to(torch.bfloat16).eval()
    ids = prompt_ids(model.config.vocab_size, args.seq_len).to(dev)
    res = quality_smoke(model, ids, args.decode_len, args.top_k)
    text = json.dumps(res, indent=1)
    if args.out_path:
        with open(args.out_path, "w") as f:
            f.write(text)
    print(json.dumps(res["metrics"]))


if __name__ == "__main__":
    main()
