"""CPU oracle for the integer transformer datapath -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy int64 arithmetic, the algorithm of llaccel's
numpy golden model (`python/llaccel/golden.py`) and of the C++ contract header
(`include/llaccel/numerics.h`).  It exists so that `tests/`, `__graft_entry__.smoke()`
and the `cpu_baseline` leg of `bench.py` can check the CUDA backend.  Nothing in the
product (`llaccel_b200/`) imports it; the CUDA path never falls back to it.

Pinning: `tests/test_oracle.py` checks every function here against the golden vectors
committed under `tests/golden/` (made by `tests/golden/make_fixtures.py` from the
reference's own golden model and quantizer) and against the reference's KATs
(tests/python/test_golden_primitives.py, test_rounding_boundaries.py).

Arithmetic notes (all exact):
* every intermediate is int64; products that the contract widens to i48/i64 stay
  below 2^63 for valid parameters (M < 2^32, S <= 63);
* `linear` uses float64 BLAS only because an i8 x i8 dot product over K < 2^38
  terms is exactly representable in a double (|sum| <= K * 2^14 < 2^53), matching the
  reference's `exact_blas_matmul` (golden.py:217-240) bit for bit.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

I64 = np.int64

# ---------------------------------------------------------------------------------------
# Look-up tables (python/llaccel/luts.py:18-29).  Generated from their definitions with
# Python's round-half-even, as the reference does; test_oracle pins them to the
# committed values in tests/golden/luts.json.
# ---------------------------------------------------------------------------------------


def sigmoid_table() -> np.ndarray:
    """SIG[j] = round(65536 * sigmoid(-8 + j/16)), j = 0..256, capped at 65535 (luts.py:18-21)."""
    out = []
    for j in range(257):
        x = j / 16.0 - 8.0
        out.append(min(65535, round(65536.0 / (1.0 + math.exp(-x)))))
    return np.array(out, dtype=I64)


def exp_int_table() -> np.ndarray:
    """EXPI[i] = round(65535 * e^-i), i = 0..15 (luts.py:24-25)."""
    return np.array([round(65535 * math.exp(-i)) for i in range(16)], dtype=I64)


def exp_frac_table() -> np.ndarray:
    """EXPF[f] = round(65535 * e^(-f/256)), f = 0..255 (luts.py:28-29)."""
    return np.array([round(65535 * math.exp(-f / 256.0)) for f in range(256)], dtype=I64)


SIG = sigmoid_table()
EXPI = exp_int_table()
EXPF = exp_frac_table()

# ---------------------------------------------------------------------------------------
# Primitives (numerics.h:15-36, golden.py:35-88, NUMERICS.md "Primitives")
# ---------------------------------------------------------------------------------------


def rshr(v, s):
    """Round-half-up arithmetic right shift; s == 0 passes v through (numerics.h:15-18).

    The rounding bit is taken before the shift so no intermediate leaves int64."""
    v = np.asarray(v, dtype=I64)
    s = np.asarray(s, dtype=I64)
    s1 = np.maximum(s, 1)
    shifted = (v >> s1) + ((v >> (s1 - 1)) & 1)
    return np.where(s == 0, v, shifted)


def sat8(v):
    return np.clip(np.asarray(v, dtype=I64), -128, 127)


def satu8(v):
    return np.clip(np.asarray(v, dtype=I64), 0, 255)


def sat16(v):
    return np.clip(np.asarray(v, dtype=I64), -32768, 32767)


def satu16(v):
    return np.clip(np.asarray(v, dtype=I64), 0, 65535)


def mulshift(v, M, S):
    """rshr(v * M, S) with the product in int64 (numerics.h:23)."""
    return rshr(np.asarray(v, dtype=I64) * np.asarray(M, dtype=I64), S)


def isqrt48(t: int) -> int:
    """floor(sqrt(t)) for 0 <= t < 2^48 (numerics.h:26-35 computes it bit-serially; the
    floor square root is unique, so math.isqrt gives the identical value)."""
    t = int(t)
    if t < 0 or t >= 1 << 48:
        raise ValueError(f"isqrt48 input out of range: {t}")
    return math.isqrt(t)


def udiv(a: int, b: int) -> int:
    """Unsigned floor division, b == 0 treated as 1, result truncated to u32 (numerics.h:36)."""
    a, b = int(a), int(b)
    if a < 0 or b < 0:
        raise ValueError("udiv operands must be unsigned")
    return (a // max(b, 1)) & 0xFFFFFFFF


def requant16(acc, M, S):
    return sat16(mulshift(acc, M, S))


def requant8(acc, M, S):
    return sat8(mulshift(acc, M, S))


def silu16(x, Mi, Si, sh_out):
    """LUT SiLU with linear interpolation between sigmoid samples (numerics.h:45-51)."""
    x = np.asarray(x, dtype=I64)
    u = sat16(mulshift(x, Mi, Si))
    idx = (u >> 8) + 128
    frac = u & 255
    lo = SIG[idx]
    sg = lo + (((SIG[idx + 1] - lo) * frac) >> 8)
    return sat16(rshr(x * sg, sh_out))


def vmul(a, b, sh):
    return sat16(rshr(np.asarray(a, dtype=I64) * np.asarray(b, dtype=I64), sh))


def vadd(a, b, sh_b):
    return sat16(np.asarray(a, dtype=I64) + rshr(b, sh_b))


def vquant(x, M, S):
    return sat8(mulshift(x, M, S))


def rmsnorm(x, g, eps_t, C, sh_post):
    """Row-wise integer RMSNorm over the last axis (numerics.h:60-71, NUMERICS.md:88-111)."""
    x = np.asarray(x, dtype=I64)
    g = np.asarray(g, dtype=I64)
    rows = x.reshape(-1, x.shape[-1])
    out = np.empty_like(rows)
    for i, row in enumerate(rows):
        ss = int(np.dot(row, row))
        r = isqrt48(ss + int(eps_t))
        inv = min(65535, udiv(C, max(r, 1)))
        out[i] = sat16(rshr(row * g * I64(inv), sh_post))
    return out.reshape(x.shape)


def rope(x, H, D, cos_tab, sin_tab, pos):
    """rotate_half RoPE with Q1.14 tables; row m uses table row pos + m (numerics.h:75-84)."""
    x = np.asarray(x, dtype=I64)
    M = x.shape[0]
    half = D // 2
    c = np.asarray(cos_tab[pos : pos + M], dtype=I64)[:, None, :]
    s = np.asarray(sin_tab[pos : pos + M], dtype=I64)[:, None, :]
    xh = x.reshape(M, H, D)
    x1, x2 = xh[..., :half], xh[..., half:]
    y1 = sat16(rshr(x1 * c - x2 * s, 14))
    y2 = sat16(rshr(x2 * c + x1 * s, 14))
    return np.concatenate([y1, y2], axis=-1).reshape(M, H * D)


def _probs(z):
    """p = z >= 4096 ? 0 : (EXPI[z>>8] * EXPF[z&255] + 2^15) >> 16 (numerics.h:104-107)."""
    zc = np.minimum(z, 4095)
    p = (EXPI[zc >> 8] * EXPF[zc & 255] + (1 << 15)) >> 16
    return np.where(z < 4096, p, 0)


def attention_head(q, keys, vals, Ms, Ss, Mo, So, prob_bits=8):
    """One query row, one head, T = len(keys) keys (numerics.h:88-120, golden.py:162-180)."""
    if prob_bits not in (8, 15):
        raise ValueError("attention prob_bits must be 8 or 15")
    q = np.asarray(q, dtype=I64)
    keys = np.asarray(keys, dtype=I64)
    vals = np.asarray(vals, dtype=I64)
    s = keys @ q
    z = mulshift(s.max() - s, Ms, Ss)
    p = _probs(z)
    inv = udiv(1 << 31, int(p.sum()))
    pn = np.minimum(rshr(p * I64(inv), 31 - prob_bits), (1 << prob_bits) - 1)
    o = pn @ vals
    if prob_bits == 15:
        o = rshr(o, 7)
    return sat8(mulshift(o, Mo, So))


def attention_rows(q, kc, vc, H, Hkv, D, pos, Ms, Ss, Mo, So, prob_bits=8):
    """Causal GQA attention for M query rows at positions pos..pos+M-1 over one sequence's
    cache kc/vc [Hkv][max_seq][D] (golden.py:353-366); vectorised over rows.

    Row m sees keys 0..pos+m; masked keys get p = 0, which leaves max, sum and the
    value sum exactly as if they were absent."""
    if prob_bits not in (8, 15):
        raise ValueError("attention prob_bits must be 8 or 15")
    q = np.asarray(q, dtype=I64)
    M = q.shape[0]
    Tm = pos + M
    rep = H // Hkv
    t_idx = np.arange(Tm)[None, :]
    valid = t_idx <= (pos + np.arange(M))[:, None]
    out = np.zeros((M, H * D), dtype=I64)
    for h in range(H):
        kvh = h // rep
        K = kc[kvh, :Tm].astype(I64)
        V = vc[kvh, :Tm].astype(I64)
        s = _exact_product(q[:, h * D : (h + 1) * D], K.T)
        mx = np.where(valid, s, np.iinfo(np.int64).min).max(axis=1, keepdims=True)
        z = mulshift(np.where(valid, mx - s, 0), Ms, Ss)
        p = np.where(valid, _probs(z), 0)
        tot = p.sum(axis=1)
        inv = np.array([udiv(1 << 31, int(t)) for t in tot], dtype=I64)[:, None]
        pn = np.minimum(rshr(p * inv, 31 - prob_bits), (1 << prob_bits) - 1)
        o = _exact_product(pn, V)
        if prob_bits == 15:
            o = rshr(o, 7)
        out[:, h * D : (h + 1) * D] = sat8(mulshift(o, Mo, So))
    return out


def _exact_product(a, b):
    """Integer a @ b, through float64 when every partial sum is below 2^53 (q.k: int8 x int8
    over D; p.v: p < 2^15 times int8 over the keys), else in int64."""
    amax = int(np.abs(a).max(initial=0))
    bmax = int(np.abs(b).max(initial=0))
    if amax * bmax * a.shape[1] < 1 << 53:
        return (a.astype(np.float64) @ b.astype(np.float64)).astype(I64)
    return a @ b


def exact_matmul(a, w, w64=None):
    """Integer A @ W.T, exact through float64 (see module docstring).  `w64`: W already
    converted to float64 (a cache; the same values)."""
    a = np.asarray(a)
    w = np.asarray(w)
    amax = int(np.abs(a.astype(I64)).max(initial=0))
    if a.shape[1] * amax * 128 >= 1 << 53:
        return a.astype(I64) @ w.astype(I64).T
    wf = w64 if w64 is not None else w.astype(np.float64)
    return (a.astype(np.float64) @ wf.T).astype(I64)


# ---------------------------------------------------------------------------------------
# Quantized graph (DIALECT.md section 2; golden.py:186-214)
# ---------------------------------------------------------------------------------------
_DTYPES = {"i8": "<i1", "i16": "<i2", "i32": "<i4", "rq": "<i4"}


class OracleGraph:
    """qgraph.json + qweights.bin, tensors as numpy views of the weight blob."""

    def __init__(self, qdir) -> None:
        self.dir = Path(qdir)
        self.g = json.loads((self.dir / "qgraph.json").read_text())
        self.model = self.g["model"]
        self.ops = self.g["ops"]
        blob = np.fromfile(self.dir / self.g["weights_file"], dtype=np.uint8)
        self.tensors: dict[str, np.ndarray] = {}
        for name, spec in self.g["tensors"].items():
            n = int(np.prod(spec["shape"]))
            dt = np.dtype(_DTYPES[spec["dtype"]])
            if spec["dtype"] == "rq":
                arr = np.frombuffer(blob, dtype=dt, count=2 * n, offset=spec["offset"]).reshape(n, 2)
            else:
                arr = np.frombuffer(blob, dtype=dt, count=n, offset=spec["offset"]).reshape(spec["shape"])
            self.tensors[name] = arr
        self.input_name = self.g.get("input", "input")
        self.output_name = self.g.get("output", "logits")


class OracleModel:
    """Mirror of GoldenModel (golden.py:246-440): same launches, same records, same errors."""

    def __init__(self, qgraph_dir) -> None:
        self.q = OracleGraph(qgraph_dir)
        m = self.q.model
        self.dim = int(m["dim"])
        self.vocab = int(m["vocab"])
        self.vocab_padded = int(m.get("vocab_padded", self.vocab))
        self.max_seq = int(m["max_seq"])
        self.prefill_m = int(m.get("prefill_m", 16))
        if not 1 <= self.prefill_m <= 16 or self.max_seq % self.prefill_m:
            raise ValueError("max_seq must be divisible by prefill_m in [1,16]")
        self.E_RES = int(m["E_RES"])
        self.E_LOGIT = int(m["E_LOGIT"])
        self.embed = self.q.tensors["embed"]
        self.rope_cos = self.q.tensors["rope_cos"]
        self.rope_sin = self.q.tensors["rope_sin"]
        # float64 copies of the int8 weights, made on first use (exact: int8 values);
        # saves re-converting large matrices (the vocabulary projection) every launch
        self._w64: dict[str, np.ndarray] = {}
        self.reset()

    def _weights64(self, name: str) -> np.ndarray:
        w = self._w64.get(name)
        if w is None:
            w = self._w64[name] = self.q.tensors[name].astype(np.float64)
        return w

    def reset(self) -> None:
        """Zero the per-layer KV caches [Hkv][max_seq][D] (golden.py:266-272)."""
        self.kv = {}
        for op in self.q.ops:
            if op["op"] == "kv_write":
                shape = (int(op["Hkv"]), self.max_seq, int(op["D"]))
                self.kv[int(op["layer"])] = (np.zeros(shape, np.int8), np.zeros(shape, np.int8))

    def _linear(self, op, act):
        """GEMM + bias + per-channel requant + epilogue (golden.py:316-342, NUMERICS.md:62-86)."""
        a = act[op["in"]]
        w = self.q.tensors[op["w"]]
        N, K = int(op["N"]), int(op["K"])
        if w.shape != (N, K) or a.shape[1] != K:
            raise ValueError(f"linear {op['out']}: shapes A{a.shape} W{w.shape} vs N={N} K={K}")
        return self._requant(op, exact_matmul(a, w, self._weights64(op["w"])), act)

    def _requant(self, op, acc, act):
        """Bias (64-bit add), per-channel requant and epilogue of an int32 accumulator
        (golden.py:325-342).  Shared by `linear` and by the tensor-parallel `requant` op,
        which applies it to the all-reduced partial accumulators."""
        rq = self.q.tensors[op["rq"]]
        if op.get("bias"):
            acc = acc + self.q.tensors[op["bias"]].astype(I64)[None, :]
        Mn = rq[:, 0].astype(I64)[None, :]
        Sn = rq[:, 1].astype(I64)[None, :]
        ep = op.get("epilogue", "none")
        if op.get("out_dtype", "i16") == "i8":
            if ep != "none":
                raise ValueError("i8 output is only valid with epilogue none")
            return requant8(acc, Mn, Sn)
        t = requant16(acc, Mn, Sn)
        if ep == "none":
            return t
        if ep == "resadd":
            return sat16(t + act[op["aux"]])
        if ep == "silu":
            s = op["silu"]
            return silu16(t, s["Mi"], s["Si"], s["sh_out"])
        if ep == "mul":
            return sat16(rshr(t * act[op["aux"]], op["aux_shift"]))
        raise ValueError(f"unknown epilogue {ep!r}")

    def run_chunk(self, rows, pos, acts=None):
        """One launch: the op list over rows [M][dim] at positions pos..pos+M-1
        (golden.py:275-314).  Returns logits [M][vocab_padded]."""
        rows = np.asarray(rows, dtype=I64)
        M = rows.shape[0]
        if pos < 0 or pos + M > self.max_seq:
            raise ValueError(f"positions {pos}..{pos + M - 1} exceed max_seq={self.max_seq}")
        act = {self.q.input_name: rows}
        for op in self.q.ops:
            self.step(op, act, pos)
        if acts is not None:
            acts.update(act)
        return act[self.q.output_name]

    def step(self, op, act, pos):
        """Execute one qgraph op on the activation dict `act` (golden.py:281-312)."""
        T = self.q.tensors
        M = act[self.q.input_name].shape[0]
        kind = op["op"]
        if kind == "rmsnorm":
            x = act[op["in"]]
            g = T[op["gamma"]]
            heads = int(op.get("heads", 1))
            if heads < 1 or x.shape[1] != heads * len(g):
                raise ValueError("RMSNorm head geometry mismatch")
            y = rmsnorm(x.reshape(-1, len(g)), g, op["eps_t"], op["C"], op["sh_post"])
            act[op["out"]] = y.reshape(x.shape)
        elif kind == "quant":
            act[op["out"]] = vquant(act[op["in"]], op["M"], op["S"])
        elif kind == "linear":
            act[op["out"]] = self._linear(op, act)
        elif kind == "linear_partial":
            # tensor parallel: this rank's K slice of a row-split linear, raw int32 sums
            a, w = act[op["in"]], T[op["w"]]
            if w.shape != (int(op["N"]), int(op["K"])) or a.shape[1] != int(op["K"]):
                raise ValueError(f"linear_partial {op['out']}: shape mismatch")
            acc = exact_matmul(a, w, self._weights64(op["w"]))
            if np.abs(acc).max(initial=0) >= 2**31:
                raise ValueError("int32 partial accumulator overflow")
            act[op["out"]] = acc
        elif kind == "requant":
            # tensor parallel: bias + requant + epilogue of the all-reduced accumulator
            act[op["out"]] = self._requant(op, act[op["in"]], act)
        elif kind == "allreduce":
            raise ValueError("allreduce needs the other ranks: run the graph with a tensor-parallel runner")
        elif kind == "rope":
            act[op["out"]] = rope(act[op["in"]], int(op["H"]), int(op["D"]), self.rope_cos, self.rope_sin, pos)
        elif kind == "kv_write":
            kc, vc = self.kv[int(op["layer"])]
            Hkv, D = int(op["Hkv"]), int(op["D"])
            k = act[op["k"]].reshape(M, Hkv, D)
            v = act[op["v"]].reshape(M, Hkv, D)
            kc[:, pos : pos + M] = k.transpose(1, 0, 2)
            vc[:, pos : pos + M] = v.transpose(1, 0, 2)
        elif kind == "attention":
            kc, vc = self.kv[int(op["layer"])]
            act[op["out"]] = attention_rows(act[op["q"]], kc, vc, int(op["H"]), int(op["Hkv"]), int(op["D"]), pos,
                                            op["Ms"], op["Ss"], op["Mo"], op["So"], op.get("prob_bits", 8))
        elif kind == "add":
            act[op["out"]] = vadd(act[op["a"]], act[op["b"]], op["sh_b"])
        elif kind == "mul":
            act[op["out"]] = vmul(act[op["a"]], act[op["b"]], op["sh"])
        elif kind == "silu":
            act[op["out"]] = silu16(act[op["in"]], op["Mi"], op["Si"], op["sh_out"])
        else:
            raise ValueError(f"unknown qgraph op {kind!r}")

    def embed_rows(self, tokens, M):
        rows = np.zeros((M, self.dim), I64)
        for i, t in enumerate(tokens):
            rows[i] = self.embed[int(t)]
        return rows

    def prefill(self, tokens, acts=None):
        tokens = [int(t) for t in tokens]
        out = []
        for start in range(0, len(tokens), self.prefill_m):
            chunk = tokens[start : start + self.prefill_m]
            a = {} if acts is not None else None
            logits = self.run_chunk(self.embed_rows(chunk, self.prefill_m), start, a)
            if acts is not None:
                acts.append({"kind": "prefill", "pos": start, "rows": self.prefill_m, "valid_rows": len(chunk), "acts": a})
            out.extend(logits[: len(chunk)])
        return out

    def decode(self, token, pos, acts=None):
        a = {} if acts is not None else None
        logits = self.run_chunk(self.embed_rows([token], 1), pos, a)
        if acts is not None:
            acts.append({"kind": "decode", "pos": pos, "rows": 1, "valid_rows": 1, "acts": a})
        return logits[0]

    def generate(self, prompt_tokens, n_tokens, acts=None):
        """Greedy generation with the runtime's launch sequence and golden.json record
        (golden.py:399-440; runtime/src/host.cpp:137-188)."""
        if not isinstance(n_tokens, int) or n_tokens < 0:
            raise ValueError("n_tokens must be a nonnegative integer")
        prompt = [int(t) for t in prompt_tokens]
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + n_tokens > self.max_seq:
            raise ValueError(f"prompt + tokens = {len(prompt) + n_tokens} exceeds max_seq={self.max_seq}")
        self.reset()
        steps, argmaxes, logit_rows = [], [], []

        def record(kind, pos, valid, row):
            steps.append({"kind": kind, "pos": pos, "rows": self.prefill_m if kind == "prefill" else 1, "valid_rows": valid})
            am = int(np.argmax(row[: self.vocab]))
            argmaxes.append(am)
            logit_rows.append([int(v) for v in row[: self.vocab]])
            return am

        rows = self.prefill(prompt, acts)
        L = len(prompt)
        nxt = -1
        for c in range(math.ceil(L / self.prefill_m)):
            last = min(L, (c + 1) * self.prefill_m) - 1
            nxt = record("prefill", c * self.prefill_m, last + 1 - c * self.prefill_m, rows[last])
        generated = []
        for i in range(n_tokens):
            generated.append(nxt)
            if L + i + 1 >= self.max_seq:
                break
            nxt = record("decode", L + i, 1, self.decode(nxt, L + i, acts))
        return {"prompt_tokens": prompt, "generated": generated, "argmax_per_step": argmaxes,
                "logits_last_rows": logit_rows, "steps": steps,
                "model": {"vocab": self.vocab, "vocab_padded": self.vocab_padded, "E_LOGIT": self.E_LOGIT,
                          "E_RES": self.E_RES, "max_seq": self.max_seq}}
