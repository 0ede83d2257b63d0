"""Quality of the integer datapath against the float model (llaccel.verify, verify.py:30-60).

The integer backend is checked bit for bit against the golden model; this module answers the
other question the reference's verify tool asks: how close the quantized model is to the
fp32 model it came from.  The fp32 model runs teacher-forced on the exact token stream the
integer model generated, so both predict each next token from the same context, and every
recorded step is compared: top-1 agreement and cosine similarity between the dequantized
i16 logits and the fp32 logits.

Dequantization is exact: an i16 logit times 2^E_LOGIT is representable in float64 (and in
float32), so the host-side float logits of this backend and of the reference agree with zero
relative error whenever the integer logits agree.
"""
from __future__ import annotations

import numpy as np


def dequantize_logits(rows, E_LOGIT: int) -> np.ndarray:
    """i16 logits -> float64 logits, value * 2^E_LOGIT (exact)."""
    return np.asarray(rows, dtype=np.int64).astype(np.float64) * (2.0 ** int(E_LOGIT))


def _cosine(a: np.ndarray, b: np.ndarray) -> float:
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 or nb == 0:
        return 0.0
    return float(np.dot(a, b) / (na * nb))


def compare_record(rec: dict, fp32_logits: np.ndarray) -> dict:
    """Per recorded step of a golden.json record: dequantized vs fp32 logits at the same
    context (step j predicts the token after pos + valid_rows tokens)."""
    vocab, E = rec["model"]["vocab"], rec["model"]["E_LOGIT"]
    rows = []
    for j, step in enumerate(rec["steps"]):
        ctx = step["pos"] + step["valid_rows"]
        gl = dequantize_logits(rec["logits_last_rows"][j][:vocab], E)
        fl = np.asarray(fp32_logits[ctx - 1])  # kept float32, as verify.py computes its norm
        rows.append({"step": j, "kind": step["kind"], "ctx": ctx, "int_top1": int(np.argmax(gl)),
                     "fp32_top1": int(np.argmax(fl)), "cos": _cosine(gl, fl)})
    return {"rows": rows, "n_steps": len(rows),
            "top1_agreement": float(np.mean([r["int_top1"] == r["fp32_top1"] for r in rows])),
            "mean_cosine": float(np.mean([r["cos"] for r in rows]))}


def teacher_forced_logits(cfg, weights: dict, tokens, device: str = "cpu") -> np.ndarray:
    """fp32 logits [T][vocab] of the architecture over `tokens` in one causal pass
    (llaccel_b200.artefacts.float_forward; weights as numpy or torch float tensors)."""
    import torch

    from . import artefacts
    W = {k: (v if isinstance(v, torch.Tensor) else torch.from_numpy(np.asarray(v, dtype=np.float32))).to(device)
         for k, v in weights.items()}
    if "lm_head" not in W:
        W["lm_head"] = W["embed"]
    for i in range(cfg.n_layers):
        for nm in ("attn_norm", "ffn_norm"):
            W.setdefault(f"l{i}_{nm}", torch.ones(cfg.dim, device=device))
    W.setdefault("norm", torch.ones(cfg.dim, device=device))
    return artefacts.float_forward(cfg, W, list(tokens), device).float().cpu().numpy()


def compare_model(model, cfg, weights: dict, prompt, n_tokens: int, device: str = "cpu") -> dict:
    """Greedy generation on `model` (CudaModel or any GoldenModel-like object), then the
    fp32 model teacher-forced on prompt + generated tokens; returns compare_record's report
    plus both token streams."""
    rec = model.generate(list(prompt), n_tokens)
    fp = teacher_forced_logits(cfg, weights, rec["prompt_tokens"] + rec["generated"], device)
    out = compare_record(rec, fp)
    out["tokens"] = rec["generated"]
    return out
