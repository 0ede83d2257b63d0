"""Test helper: hand-built qgraphs with random integer weights and parameters spanning the
numeric ranges the contract allows (full-range int8 weights, saturating requant shifts,
large biases, tiny and huge RMS rows), in the style of the reference's own compiler-free
fixture (tests/python/test_golden_e2e.py build_fixture).  The graphs are not calibrated
models; they exist to drive every kernel path through its saturation and rounding edges.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np


class _Blob:
    def __init__(self):
        self.parts, self.off, self.tensors = [], 0, {}

    def add(self, name, arr, dtype, exp=None):
        raw = np.ascontiguousarray(np.asarray(arr).astype({"i8": "<i1", "i16": "<i2", "i32": "<i4", "rq": "<i4"}[dtype]))
        shape = list(arr.shape[:-1]) if dtype == "rq" else list(arr.shape)
        spec = {"dtype": dtype, "shape": [int(s) for s in shape], "offset": self.off}
        if exp is not None:
            spec["exp"] = exp
        self.tensors[name] = spec
        b = raw.tobytes()
        b += b"\0" * ((-len(b)) % 64)
        self.parts.append(b)
        self.off += len(b)


def build(out: Path, *, dim=64, n_layers=2, H=4, Hkv=2, D=32, ffn=96, vocab=40, max_seq=64, fuse=True, seed=0,
          qk_norm=False, bias=True, prob_bits=15, extreme=False, prefill_m=16, att_S=(28, 41)) -> Path:
    rng = np.random.default_rng(seed)
    vp = (vocab + 15) // 16 * 16
    blob = _Blob()
    ops = []
    amp = 32767 if extreme else 9000
    emb = rng.integers(-amp, amp + 1, (vp, dim))
    emb[vocab:] = 0
    blob.add("embed", emb, "i16", -10)
    inv = 10000.0 ** (-np.arange(0, D, 2) / D)
    ang = np.outer(np.arange(max_seq), inv)
    blob.add("rope_cos", np.round(np.cos(ang) * 16384).astype(np.int16), "i16")
    blob.add("rope_sin", np.round(np.sin(ang) * 16384).astype(np.int16), "i16")

    def rq_table(N, lo_s, hi_s):
        M = rng.integers(1 << 30, 1 << 31, N)
        S = rng.integers(lo_s, hi_s, N)
        return np.stack([M, S], 1)

    def rms(x, g, y, K, heads=1):
        blob.add(g, rng.integers(4000, 32767, K), "i16", -14)
        R = int(rng.integers(22, 28))
        op = {"op": "rmsnorm", "in": x, "gamma": g, "out": y, "K": K,
              "eps_t": int(rng.integers(0, 1 << 20)), "C": int(round(2.0**R * math.sqrt(K))),
              "sh_post": int(R + int(rng.integers(-2, 4)))}
        if heads != 1:
            op["heads"] = heads
        ops.append(op)

    def quant(x):
        ops.append({"op": "quant", "in": x, "out": x + ".q", "M": int(rng.integers(1 << 30, 1 << 31)),
                    "S": int(rng.integers(35, 41))})
        return x + ".q"

    def lin(a, w, y, N, K, out_dtype="i16", ep="none", aux=None, aux_shift=0, silu=None, has_bias=False):
        blob.add(w, rng.integers(-128, 128, (N, K)), "i8")
        lo, hi = (30, 38) if out_dtype == "i16" else (34, 42)
        if extreme:
            lo, hi = lo - 6, hi - 4
        blob.add(w + ".rq", rq_table(N, lo, hi), "rq")
        b = None
        if has_bias:
            lim = 1 << 24 if extreme else 1 << 14
            blob.add(w + ".b", rng.integers(-lim, lim, N), "i32")
            b = w + ".b"
        ops.append({"op": "linear", "in": a, "w": w, "rq": w + ".rq", "bias": b, "out": y, "N": N, "K": K,
                    "out_dtype": out_dtype, "epilogue": ep, "aux": aux, "aux_shift": aux_shift, "silu": silu})

    resid = "input"
    for i in range(n_layers):
        p = f"l{i}"
        rms(resid, f"{p}_attn_norm", f"{p}.h", dim)
        hq = quant(f"{p}.h")
        lin(hq, f"{p}_wq", f"{p}.q", H * D, dim, has_bias=bias)
        lin(hq, f"{p}_wk", f"{p}.k", Hkv * D, dim, has_bias=bias)
        lin(hq, f"{p}_wv", f"{p}.v", Hkv * D, dim, "i8", has_bias=bias)
        qs, ks = f"{p}.q", f"{p}.k"
        if qk_norm:
            rms(f"{p}.q", f"{p}_q_norm", f"{p}.qn", D, heads=H)
            rms(f"{p}.k", f"{p}_k_norm", f"{p}.kn", D, heads=Hkv)
            qs, ks = f"{p}.qn", f"{p}.kn"
        ops.append({"op": "rope", "in": qs, "out": f"{p}.qr", "H": H, "D": D})
        ops.append({"op": "rope", "in": ks, "out": f"{p}.kr", "H": Hkv, "D": D})
        qq, kq = quant(f"{p}.qr"), quant(f"{p}.kr")
        ops.append({"op": "kv_write", "layer": i, "k": kq, "v": f"{p}.v", "Hkv": Hkv, "D": D})
        ops.append({"op": "attention", "q": qq, "layer": i, "out": f"{p}.a", "H": H, "Hkv": Hkv, "D": D,
                    "Ms": int(rng.integers(1 << 30, 1 << 31)), "Ss": int(rng.integers(*att_S)),
                    "Mo": int(rng.integers(1 << 30, 1 << 31)), "So": int(rng.integers(36, 40)),
                    "prob_bits": prob_bits})
        silu = {"Mi": int(rng.integers(1 << 30, 1 << 32)), "Si": int(rng.integers(28, 38)),
                "sh_out": int(rng.integers(14, 19))}
        sh_mul = int(rng.integers(12, 17))
        if fuse:
            lin(f"{p}.a", f"{p}_wo", f"{p}.x1", dim, H * D, ep="resadd", aux=resid)
        else:
            lin(f"{p}.a", f"{p}_wo", f"{p}.o", dim, H * D)
            ops.append({"op": "add", "a": resid, "b": f"{p}.o", "out": f"{p}.x1", "sh_b": int(rng.integers(0, 3))})
        rms(f"{p}.x1", f"{p}_ffn_norm", f"{p}.h2", dim)
        h2q = quant(f"{p}.h2")
        if fuse:
            lin(h2q, f"{p}_wg", f"{p}.sg", ffn, dim, ep="silu", silu=silu)
            lin(h2q, f"{p}_wu", f"{p}.f", ffn, dim, ep="mul", aux=f"{p}.sg", aux_shift=sh_mul)
        else:
            lin(h2q, f"{p}_wg", f"{p}.g", ffn, dim)
            lin(h2q, f"{p}_wu", f"{p}.u", ffn, dim)
            ops.append({"op": "silu", "in": f"{p}.g", "out": f"{p}.sg", **silu})
            ops.append({"op": "mul", "a": f"{p}.sg", "b": f"{p}.u", "out": f"{p}.f", "sh": sh_mul})
        fq = quant(f"{p}.f")
        if fuse:
            lin(fq, f"{p}_wd", f"{p}.x2", dim, ffn, ep="resadd", aux=f"{p}.x1")
        else:
            lin(fq, f"{p}_wd", f"{p}.d", dim, ffn)
            ops.append({"op": "add", "a": f"{p}.x1", "b": f"{p}.d", "out": f"{p}.x2", "sh_b": 0})
        resid = f"{p}.x2"
    rms(resid, "norm", "hn", dim)
    hnq = quant("hn")
    lin(hnq, "lm_head", "logits", vp, dim)
    g = {"model": {"dim": dim, "n_layers": n_layers, "n_heads": H, "n_kv_heads": Hkv, "head_dim": D, "ffn": ffn,
                   "vocab": vocab, "vocab_padded": vp, "max_seq": max_seq, "E_RES": -10, "E_LOGIT": -6,
                   "prefill_m": prefill_m},
         "weights_file": "qweights.bin", "tensors": blob.tensors, "ops": ops, "input": "input", "output": "logits"}
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    (out / "qweights.bin").write_bytes(b"".join(blob.parts))
    (out / "qgraph.json").write_text(json.dumps(g))
    return out


def build_linear(out: Path, *, K: int, N: int, epi: str = "none", chain_i8: int = 0, seed: int = 0,
                 bias: bool = True, max_seq: int = 512) -> Path:
    """Minimal graph: quant(input) -> [linear i8 out (chain_i8 channels) ->] linear -> logits.
    epi selects the final linear's epilogue (resadd/mul use `input` as aux, so N == K there)."""
    rng = np.random.default_rng(seed)
    blob = _Blob()
    dim = K
    blob.add("embed", rng.integers(-20000, 20000, (16, dim)), "i16", -10)
    blob.add("rope_cos", np.zeros((max_seq, 8), np.int16), "i16")
    blob.add("rope_sin", np.zeros((max_seq, 8), np.int16), "i16")
    ops = [{"op": "quant", "in": "input", "out": "input.q", "M": int(rng.integers(1 << 30, 1 << 31)), "S": 37}]

    def lin(a, w, y, n, k, out_dtype, ep, aux=None, aux_shift=0, silu=None):
        blob.add(w, rng.integers(-128, 128, (n, k)), "i8")
        lo, hi = (26, 36) if out_dtype == "i16" else (30, 40)
        blob.add(w + ".rq", np.stack([rng.integers(1 << 30, 1 << 31, n), rng.integers(lo, hi, n)], 1), "rq")
        b = None
        if bias:
            blob.add(w + ".b", rng.integers(-(1 << 20), 1 << 20, n), "i32")
            b = w + ".b"
        ops.append({"op": "linear", "in": a, "w": w, "rq": w + ".rq", "bias": b, "out": y, "N": n, "K": k,
                    "out_dtype": out_dtype, "epilogue": ep, "aux": aux, "aux_shift": aux_shift, "silu": silu})

    src, k = "input.q", K
    if chain_i8:
        lin(src, "w0", "mid", chain_i8, K, "i8", "none")
        src, k = "mid", chain_i8
    kw = {}
    if epi in ("resadd", "mul"):
        assert N == K
        kw = {"aux": "input", "aux_shift": 15 if epi == "mul" else 0}
    if epi == "silu":
        kw = {"silu": {"Mi": 1 << 30, "Si": 30, "sh_out": 16}}
    lin(src, "w1", "logits", N, k, "i16", epi, **kw)
    g = {"model": {"dim": dim, "n_layers": 0, "n_heads": 1, "n_kv_heads": 1, "head_dim": 16, "ffn": 16,
                   "vocab": min(16, N), "vocab_padded": N, "max_seq": max_seq, "E_RES": -10, "E_LOGIT": -6},
         "weights_file": "qweights.bin", "tensors": blob.tensors, "ops": ops, "input": "input", "output": "logits"}
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    (out / "qweights.bin").write_bytes(b"".join(blob.parts))
    (out / "qgraph.json").write_text(json.dumps(g))
    return out
