"""Artefact generator: random-init dense Llama/Qwen model -> `qgraph.json` + `qweights.bin`.

The CUDA backend consumes the quantized artefacts that llaccel's importer and quantizer
produce (DIALECT.md section 2).  The GPU box has no copy of llaccel, and the bench configs
go up to 8B parameters, so this module produces those artefacts itself:

1. float weights N(0, 0.02) (biases zero unless a bias std is given, norm weights one) --
   the initialisation of python/llaccel/model.py:163-170 -- generated with a seeded torch
   generator on any device;
2. a float32 forward pass of the same architecture (model.py:70-180: RMSNorm, rotate-half
   RoPE, causal GQA SDPA, SwiGLU) over uniform-random token sequences, recording the
   per-activation abs-max and RMSNorm-input RMS minimum that calibrate.py:95-133 records;
3. the quantization decisions of python/llaccel/refquant.py (restated below, each
   function citing the line it follows), emitting the same op list and tensor blob.

Given the reference exporter's float weights and calib.json, `quantize()` reproduces
refquant's output exactly (pinned by tests/test_artefacts.py against committed C1
fixtures).  Unlike refquant.py:411-412 it accepts head_dim 128, as the compiler does
(compiler/lib/Transforms/Quantize.cpp:148-149 accepts 16..256).
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np

INT32_MAX, INT32_MIN = 2**31 - 1, -(2**31)


# ---------------------------------------------------------------------------------------
# Architectures of the five benchmark configs C1..C5 (tiny Llama, SmolLM2-135M, Qwen2.5-0.5B,
# Qwen3-0.6B, Llama-3-8B), random-initialised
# ---------------------------------------------------------------------------------------
@dataclass
class ArchConfig:
    name: str
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    max_seq: int
    rope_base: float = 10000.0
    rms_eps: float = 1e-5
    qkv_bias: bool = False
    qk_norm: bool = False
    tied: bool = False
    bias_std: float = 0.0
    extra: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


def _ceil_to(x: int, m: int) -> int:
    return (x + m - 1) // m * m


CONFIGS = {
    # tiny dense Llama (seed 0), P=16 + 64 decode, context limit 256 -> max_seq 80
    "c1": ArchConfig("c1", 128, 2, 4, 2, 32, 352, 512, 80, 10000.0, 1e-5),
    # SmolLM2-135M architecture: P=128 + 128 decode -> max_seq 256
    "c2": ArchConfig("c2", 576, 30, 9, 3, 64, 1536, 49152, 256, 10000.0, 1e-5, tied=True),
    # Qwen2.5-0.5B architecture with QKV bias N(0, 0.02): P=512 + 256 decode -> 768
    "c3": ArchConfig("c3", 896, 24, 14, 2, 64, 4864, 151936, 768, 1e6, 1e-5, qkv_bias=True, tied=True,
                     bias_std=0.02),
    # Qwen3-0.6B architecture with per-head Q/K RMSNorm: P=4096 + 128 decode -> 4224
    "c4": ArchConfig("c4", 1024, 28, 16, 8, 128, 3072, 151936, 4224, 1e6, 1e-5, qk_norm=True, tied=True),
    # Llama-3-8B architecture: P=1024 + 256 decode -> 1280
    "c5": ArchConfig("c5", 4096, 32, 32, 8, 128, 14336, 128256, 1280, 5e5, 1e-5),
}

# Workload of each config: sequences per GPU, prompt tokens, greedy decode tokens.
WORKLOADS = {
    "c1": {"batch": 1, "prompt": 16, "decode": 64},
    "c2": {"batch": 32, "prompt": 128, "decode": 128},
    "c3": {"batch": 128, "prompt": 512, "decode": 256},
    "c4": {"batch": 64, "prompt": 4096, "decode": 128},
    "c5": {"batch": 256, "prompt": 1024, "decode": 256},
}


# ---------------------------------------------------------------------------------------
# Float -> int rounding and scale rules (refquant.py:61-238, QuantParams.h twins)
# ---------------------------------------------------------------------------------------
def llround(x: float) -> int:
    """C llround: nearest, halves away from zero (refquant.py:61-72)."""
    x = float(x)
    if not math.isfinite(x):
        raise ValueError(f"llround of {x}")
    t = math.trunc(x)
    d = x - t
    return t + 1 if d >= 0.5 else t - 1 if d <= -0.5 else t


def llround_np(x: np.ndarray) -> np.ndarray:
    """Vectorised llround over float64 (refquant.py:75-83)."""
    x = np.asarray(x, dtype=np.float64)
    if not np.all(np.isfinite(x)):
        raise ValueError("llround requires finite values")
    t = np.trunc(x)
    d = x - t
    return np.where(d >= 0.5, t + 1, np.where(d <= -0.5, t - 1, t)).astype(np.int64)


def normalize_mulshift(r: float) -> tuple[int, int]:
    """(M, S) with M * 2^-S ~= r, M in [2^30, 2^31) via frexp (refquant.py:89-104)."""
    if not (r > 0.0) or not math.isfinite(r):
        raise ValueError("normalize_mulshift: ratio must be positive and finite")
    f, e = math.frexp(r)
    M, S = llround(math.ldexp(f, 31)), 31 - e
    if M >= 1 << 31:
        M, S = 1 << 30, S - 1
    if S < 0:
        raise ValueError(f"normalize_mulshift: ratio {r} too large (S < 0)")
    if S > 63:
        M, S = llround(math.ldexp(r, 63)), 63
    return M, S


def normalize_mulshift_np(r: np.ndarray) -> np.ndarray:
    """Vectorised normalize_mulshift -> int64 [n][2]; identical to the scalar rule."""
    r = np.asarray(r, dtype=np.float64)
    if not np.all((r > 0) & np.isfinite(r)):
        raise ValueError("normalize_mulshift: ratio must be positive and finite")
    f, e = np.frexp(r)
    M = llround_np(np.ldexp(f, 31))
    S = 31 - e.astype(np.int64)
    up = M >= (1 << 31)
    M = np.where(up, 1 << 30, M)
    S = np.where(up, S - 1, S)
    if np.any(S < 0):
        raise ValueError("normalize_mulshift: ratio too large (S < 0)")
    tiny = S > 63
    if np.any(tiny):
        M = M.copy()
        M[tiny] = llround_np(np.ldexp(r[tiny], 63))
        S = np.where(tiny, 63, S)
    return np.stack([M, S], axis=1).astype(np.int64)


def i16_exponent(absmax: float) -> int:
    """e = max(ceil(log2(absmax / 32767)), -15), zero range -> -15 (refquant.py:107-111)."""
    if not (absmax > 0.0):
        return -15
    return max(int(math.ceil(math.log2(absmax) - math.log2(32767.0))), -15)


def i8_scale(absmax: float) -> float:
    """absmax / 127, zero range -> 1 (refquant.py:114-116)."""
    return absmax / 127.0 if absmax > 0.0 else 1.0


def quant_i16(v: np.ndarray, e: int) -> np.ndarray:
    """llround(clip(v * 2^-e)) -> i16 (refquant.py:128-134)."""
    v = np.asarray(v, dtype=np.float64)
    with np.errstate(over="ignore"):
        scaled = np.clip(np.ldexp(v, -int(e)), -32768, 32767)
    return llround_np(scaled).astype(np.int16)


def rmsnorm_params(K, eps, e_x, e_g, e_y, absmax_x, name, rms_min=None) -> dict:
    """eps_t, C, R, sh_post (refquant.py:159-186; NUMERICS.md:100-110)."""
    if rms_min is not None and (not math.isfinite(rms_min) or not 0 <= rms_min <= absmax_x):
        raise ValueError(f"rmsnorm {name}: rms_min must be finite and in [0, absmax]")
    eps_t = llround(eps * float(K) * math.ldexp(1.0, int(-2 * e_x)))
    if not 0 <= eps_t < 2**32:
        raise ValueError(f"rmsnorm {name}: eps_t does not fit u32")
    rms_q = (absmax_x / 4.0 if rms_min is None else rms_min) / math.ldexp(1.0, int(e_x))
    r_typ = max(1.0, math.floor(math.sqrt(float(K) * rms_q * rms_q + float(eps_t))))
    R = C = -1
    for cand in range(31, -1, -1):
        c = llround(math.ldexp(math.sqrt(float(K)), cand))
        if c >= 4294967296:
            continue
        if math.floor(c / r_typ) < 65535.0 / 4.0:
            R, C = cand, c
            break
    if R < 0:
        raise ValueError(f"rmsnorm {name}: no R in [0,31] keeps inv below 65535/4")
    sh_post = R - e_g + e_y
    if not 0 <= sh_post <= 63:
        raise ValueError(f"rmsnorm {name}: sh_post = {sh_post} outside [0, 63]")
    return {"eps_t": eps_t, "C": C, "R": R, "sh_post": sh_post}


def silu_params(e_x: int, e_y: int, name: str) -> dict:
    """Mi = 2^30, Si = 30 - (e_x + 12), sh_out = 16 + e_y - e_x (refquant.py:189-196)."""
    Mi, Si, sh_out = 1 << 30, 30 - (e_x + 12), 16 + e_y - e_x
    if not 0 <= Si <= 63 or not 0 <= sh_out <= 63:
        raise ValueError(f"silu {name}: shift outside [0, 63]")
    return {"Mi": Mi, "Si": Si, "sh_out": sh_out}


def mul_shift(e_a: int, e_b: int, e_y: int, name: str) -> int:
    """MUL right shift sh = e_y - e_a - e_b (refquant.py:199-209; DIALECT.md 4.2)."""
    sh = e_y - e_a - e_b
    if not 0 <= sh <= 63:
        raise ValueError(f"mul {name}: sh = {sh} outside [0, 63]")
    return sh


def add_shift(e_a: int, e_b: int, name: str) -> int:
    """ADD shift of the finer operand sh_b = e_a - e_b (refquant.py:212-218)."""
    sh = e_a - e_b
    if not 0 <= sh <= 63:
        raise ValueError(f"add {name}: sh_b = {sh} outside [0, 63]")
    return sh


def attn_params(s_q: float, s_k: float, s_v: float, s_out: float, D: int) -> dict:
    """Score and output multipliers (refquant.py:221-224; NUMERICS.md:179)."""
    Ms, Ss = normalize_mulshift(256.0 * s_q * s_k / math.sqrt(float(D)))
    Mo, So = normalize_mulshift(s_v / (256.0 * s_out))
    return {"Ms": Ms, "Ss": Ss, "Mo": Mo, "So": So}


def rope_tables(max_seq: int, D: int, base: float) -> tuple[np.ndarray, np.ndarray]:
    """Q1.14 tables llround(2^14 cos/sin(p * base^(-2i/D))) (refquant.py:227-238).  libm's
    math.cos/sin are used element by element so the rounding matches the reference."""
    half = D // 2
    cos_t = np.zeros((max_seq, half), dtype=np.int16)
    sin_t = np.zeros((max_seq, half), dtype=np.int16)
    for i in range(half):
        theta = math.pow(base, -2.0 * float(i) / float(D))
        cos_t[:, i] = [min(llround(16384.0 * math.cos(float(p) * theta)), 32767) for p in range(max_seq)]
        sin_t[:, i] = [min(llround(16384.0 * math.sin(float(p) * theta)), 32767) for p in range(max_seq)]
    return cos_t, sin_t


class TensorBlob:
    """qweights.bin writer: tensors back to back, each padded to 64 bytes; records the
    DIALECT.md `tensors` entries (layout of refquant.py:244-269)."""

    def __init__(self, path: Path | None = None) -> None:
        self.tensors: dict[str, dict] = {}
        self.off = 0
        self.fh = open(path, "wb") if path is not None else None
        self.parts: list[bytes] = []

    def add(self, name: str, arr: np.ndarray, dtype: str, exp: int | None = None) -> None:
        if name in self.tensors:
            raise ValueError(f"duplicate tensor {name}")
        np_dt = {"i8": "<i1", "i16": "<i2", "i32": "<i4", "rq": "<i4"}[dtype]
        raw = np.ascontiguousarray(np.asarray(arr).astype(np_dt)).tobytes()
        shape = list(arr.shape[:-1]) if dtype == "rq" else list(arr.shape)
        spec = {"dtype": dtype, "shape": [int(s) for s in shape], "offset": self.off}
        if exp is not None:
            spec["exp"] = int(exp)
        self.tensors[name] = spec
        pad = (-len(raw)) % 64
        chunk = raw + b"\0" * pad
        if self.fh is not None:
            self.fh.write(chunk)
        else:
            self.parts.append(chunk)
        self.off += len(chunk)

    def close(self) -> None:
        if self.fh is not None:
            self.fh.close()
            self.fh = None

    def bytes(self) -> bytes:
        return b"".join(self.parts)


# ---------------------------------------------------------------------------------------
# The quantizer (decisions of refquant.py:304-490)
# ---------------------------------------------------------------------------------------
class WeightSource:
    """Name -> float weight, fetched lazily (numpy float64 or a torch tensor)."""

    def __init__(self, weights: dict) -> None:
        self.w = weights

    def __contains__(self, name: str) -> bool:
        return name in self.w

    def get(self, name: str):
        return self.w[name]


def _to_np64(t) -> np.ndarray:
    if isinstance(t, np.ndarray):
        return t.astype(np.float64, copy=False)
    return t.detach().double().cpu().numpy()


def _quant_weight_rows(w):
    """Per-output-channel int8: s[n] = max|W[n,:]| / 127 (zero rows -> 1),
    q = llround(clip(W / s, -128, 127)) in float64 (refquant.py:119-140).
    Accepts numpy or torch; torch tensors are quantized on their own device in float64."""
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(w, torch.Tensor):
        wd = w.double()
        mx = wd.abs().amax(dim=1)
        s = torch.where(mx > 0, mx / 127.0, torch.ones_like(mx))
        x = torch.clamp(wd / s[:, None], -128, 127)
        t = torch.trunc(x)
        d = x - t
        q = torch.where(d >= 0.5, t + 1, torch.where(d <= -0.5, t - 1, t)).to(torch.int8)
        return q.cpu().numpy(), s.cpu().numpy()
    wd = np.asarray(w, dtype=np.float64)
    mx = np.abs(wd).max(axis=1)
    s = np.where(mx > 0.0, mx / 127.0, 1.0)
    with np.errstate(over="ignore"):
        x = np.clip(wd / s[:, None], -128, 127)
    return llround_np(x).astype(np.int8), s


class Quantizer:
    def __init__(self, cfg: dict, weights: dict, calib: dict, fusion: bool, blob: TensorBlob) -> None:
        self.cfg, self.W, self.calib, self.fusion = cfg, WeightSource(weights), calib, fusion
        self.blob = blob
        self.ops: list[dict] = []
        self.exps: dict[str, int] = {}
        self.scales: dict[str, float] = {}

    # activation formats (refquant.py:313-338)
    def absmax(self, name: str) -> float:
        if name not in self.calib:
            raise KeyError(f"calibration has no entry for activation {name!r}")
        v = float(self.calib[name])
        if not math.isfinite(v) or v < 0:
            raise ValueError(f"calibration for {name!r} must be finite and nonnegative")
        return v

    def qabsmax(self, name: str, bits: int) -> float:
        raw = self.absmax(name)
        key = f"{name}.i{bits}_absmax"
        bound = self.absmax(key) if key in self.calib else raw
        if bound > raw or (raw > 0 and bound == 0):
            raise ValueError(f"invalid selected quantization bound for {name!r}")
        return bound

    def e16(self, name: str) -> int:
        if name not in self.exps:
            self.exps[name] = i16_exponent(self.qabsmax(name, 16))
        return self.exps[name]

    def s8(self, name: str, src: str | None = None) -> float:
        if name not in self.scales:
            self.scales[name] = i8_scale(self.qabsmax(src or name.removesuffix(".q"), 8))
        return self.scales[name]

    # op emitters (refquant.py:341-400)
    def rmsnorm(self, x: str, gamma: str, y: str, heads: int = 1) -> None:
        e_x, e_y = self.e16(x), self.e16(y)
        g = _to_np64(self.W.get(gamma))
        e_g = i16_exponent(float(np.abs(g).max()))
        self.blob.add(gamma, quant_i16(g, e_g), "i16", e_g)
        K = int(g.shape[0])
        rms_min = self.absmax(x + ".rms_min") if x + ".rms_min" in self.calib else None
        p = rmsnorm_params(K, self.cfg["rms_eps"], e_x, e_g, e_y, self.absmax(x), y, rms_min)
        op = {"op": "rmsnorm", "in": x, "gamma": gamma, "out": y, "K": K, "eps_t": p["eps_t"], "C": p["C"],
              "sh_post": p["sh_post"]}
        if heads != 1:
            op["heads"] = heads
        self.ops.append(op)

    def quant(self, x: str) -> str:
        y = x + ".q"
        r = math.ldexp(1.0, int(self.e16(x))) / self.s8(y, x)
        M, S = normalize_mulshift(r)
        self.ops.append({"op": "quant", "in": x, "out": y, "M": M, "S": S})
        return y

    def linear(self, a, w, b, y, out_dtype, *, e_rq=None, N_pad=None, epilogue="none", aux=None, aux_shift=0,
               silu=None) -> None:
        wf = self.W.get(w)
        q, s_w = _quant_weight_rows(wf)
        if N_pad is not None and N_pad != q.shape[0]:
            # zero rows: scale 1, all-zero int8 (refquant pads the float matrix first)
            q = np.concatenate([q, np.zeros((N_pad - q.shape[0], q.shape[1]), np.int8)], axis=0)
            s_w = np.concatenate([s_w, np.ones(N_pad - s_w.shape[0])])
        N, K = q.shape
        self.blob.add(w, q, "i8")
        del q
        s_a = self.s8(a)
        if out_dtype == "i16":
            e_out = self.e16(y) if e_rq is None else e_rq
            r = (s_a * s_w) / math.ldexp(1.0, int(e_out))
        elif out_dtype == "i8":
            if epilogue != "none":
                raise ValueError(f"linear {y}: i8 output is only valid with epilogue none")
            r = (s_a * s_w) / self.s8(y)
        else:
            raise ValueError(out_dtype)
        self.blob.add(w + ".rq", normalize_mulshift_np(r), "rq")
        bias = None
        if b is not None and b in self.W:
            bf = _to_np64(self.W.get(b))
            bq = np.zeros(N)
            bq[: bf.shape[0]] = bf
            bi = llround_np(bq / (s_a * s_w))
            self.blob.add(b, np.clip(bi, INT32_MIN, INT32_MAX).astype(np.int32), "i32")
            bias = b
        self.ops.append({"op": "linear", "in": a, "w": w, "rq": w + ".rq", "bias": bias, "out": y, "N": int(N),
                         "K": int(K), "out_dtype": out_dtype, "epilogue": epilogue, "aux": aux,
                         "aux_shift": aux_shift, "silu": silu})

    def residual_linear(self, a, w, bias, branch, residual, out) -> None:
        e_res = self.e16(residual)
        e_br = max(self.e16(branch), self.e16(out), e_res, i16_exponent(self.qabsmax(residual, 16)))
        self.exps[branch] = self.exps[out] = e_br
        if self.fusion and e_br == e_res:
            self.linear(a, w, bias, out, "i16", e_rq=e_br, epilogue="resadd", aux=residual, aux_shift=0)
        else:
            self.linear(a, w, bias, branch, "i16")
            first, second = (residual, branch) if e_res == e_br else (branch, residual)
            self.ops.append({"op": "add", "a": first, "b": second, "out": out,
                             "sh_b": add_shift(self.e16(first), self.e16(second), out)})

    # the graph (refquant.py:403-490)
    def run(self) -> dict:
        c = self.cfg
        dim, L, H, Hkv, D, ffn, vocab, max_seq = (int(c[k]) for k in ("dim", "n_layers", "n_heads", "n_kv_heads",
                                                                    "head_dim", "ffn", "vocab", "max_seq"))
        vocab_padded = _ceil_to(vocab, 16)
        for what, val in (("dim", dim), ("ffn", ffn), ("n_kv_heads*head_dim", Hkv * D)):
            if val % 16:
                raise ValueError(f"{what} = {val} must be a multiple of 16")
        if D not in (16, 32, 64, 128, 256) or H % Hkv:
            raise ValueError(f"unsupported head geometry H={H} Hkv={Hkv} D={D}")
        E_RES = self.e16("input")
        E_LOGIT = i16_exponent(self.qabsmax("logits", 16))
        self.exps["logits"] = E_LOGIT
        emb = _to_np64(self.W.get("embed"))
        embp = np.zeros((vocab_padded, dim))
        embp[:vocab] = emb
        self.blob.add("embed", quant_i16(embp, E_RES), "i16", E_RES)
        del emb, embp
        if "rope_cos_input" in self.W or "rope_sin_input" in self.W:
            # static (scaled) RoPE tables exported as floats (refquant.py:424-431)
            tabs = []
            for nm in ("rope_cos_input", "rope_sin_input"):
                t = _to_np64(self.W.get(nm))
                if t.shape != (max_seq, D // 2) or not np.isfinite(t).all() or ((t < -2.0) | (t > 32767.0 / 16384.0)).any():
                    raise ValueError(f"invalid static RoPE table {nm}")
                tabs.append(llround_np(t * 16384.0).astype(np.int16))
            cos_t, sin_t = tabs
        else:
            cos_t, sin_t = rope_tables(max_seq, D, float(c["rope_base"]))
        self.blob.add("rope_cos", cos_t, "i16")
        self.blob.add("rope_sin", sin_t, "i16")
        residual = "input"
        for i in range(L):
            p = f"l{i}"
            self.rmsnorm(residual, f"{p}_attn_norm", f"{p}.h")
            hq = self.quant(f"{p}.h")
            qk_norm = f"{p}_q_norm" in self.W
            if qk_norm != (f"{p}_k_norm" in self.W):
                raise ValueError("Q/K normalization must be paired")
            q_src, k_src = (f"{p}.qn", f"{p}.kn") if qk_norm else (f"{p}.q", f"{p}.k")
            for a, b in ((q_src, f"{p}.qr"), (k_src, f"{p}.kr")):
                self.exps[a] = self.exps[b] = max(i16_exponent(self.qabsmax(a, 16)), i16_exponent(self.qabsmax(b, 16)))
            self.linear(hq, f"{p}_wq", f"{p}_bq", f"{p}.q", "i16")
            self.linear(hq, f"{p}_wk", f"{p}_bk", f"{p}.k", "i16")
            self.linear(hq, f"{p}_wv", f"{p}_bv", f"{p}.v", "i8")
            if qk_norm:
                self.rmsnorm(f"{p}.q", f"{p}_q_norm", q_src, heads=H)
                self.rmsnorm(f"{p}.k", f"{p}_k_norm", k_src, heads=Hkv)
            self.ops.append({"op": "rope", "in": q_src, "out": f"{p}.qr", "H": H, "D": D})
            self.ops.append({"op": "rope", "in": k_src, "out": f"{p}.kr", "H": Hkv, "D": D})
            qq, kq = self.quant(f"{p}.qr"), self.quant(f"{p}.kr")
            self.ops.append({"op": "kv_write", "layer": i, "k": kq, "v": f"{p}.v", "Hkv": Hkv, "D": D})
            self.ops.append({"op": "attention", "q": qq, "layer": i, "out": f"{p}.a", "H": H, "Hkv": Hkv, "D": D,
                             "prob_bits": 15,
                             **attn_params(self.s8(qq), self.s8(kq), self.s8(f"{p}.v"), self.s8(f"{p}.a"), D)})
            self.residual_linear(f"{p}.a", f"{p}_wo", f"{p}_bo", f"{p}.o", residual, f"{p}.x1")
            self.rmsnorm(f"{p}.x1", f"{p}_ffn_norm", f"{p}.h2")
            h2q = self.quant(f"{p}.h2")
            e_g, e_u, e_sg, e_f = (self.e16(f"{p}.{n}") for n in ("g", "u", "sg", "f"))
            silu = silu_params(e_g, e_sg, f"{p}.sg")
            sh_mul = mul_shift(e_sg, e_u, e_f, f"{p}.f")
            if self.fusion:
                self.linear(h2q, f"{p}_wg", f"{p}_bg", f"{p}.sg", "i16", e_rq=e_g, epilogue="silu", silu=silu)
                self.linear(h2q, f"{p}_wu", f"{p}_bu", f"{p}.f", "i16", e_rq=e_u, epilogue="mul", aux=f"{p}.sg",
                            aux_shift=sh_mul)
            else:
                self.linear(h2q, f"{p}_wg", f"{p}_bg", f"{p}.g", "i16")
                self.linear(h2q, f"{p}_wu", f"{p}_bu", f"{p}.u", "i16")
                self.ops.append({"op": "silu", "in": f"{p}.g", "out": f"{p}.sg", **silu})
                self.ops.append({"op": "mul", "a": f"{p}.sg", "b": f"{p}.u", "out": f"{p}.f", "sh": sh_mul})
            fq = self.quant(f"{p}.f")
            self.residual_linear(fq, f"{p}_wd", f"{p}_bd", f"{p}.d", f"{p}.x1", f"{p}.x2")
            residual = f"{p}.x2"
        self.rmsnorm(residual, "norm", "hn")
        hnq = self.quant("hn")
        self.linear(hnq, "lm_head", "lm_head_bias", "logits", "i16", N_pad=vocab_padded)
        return {
            "model": {"dim": dim, "n_layers": L, "n_heads": H, "n_kv_heads": Hkv, "head_dim": D, "ffn": ffn,
                      "vocab": vocab, "vocab_padded": vocab_padded, "max_seq": max_seq, "E_RES": E_RES,
                      "E_LOGIT": E_LOGIT},
            "weights_file": "qweights.bin",
            "tensors": self.blob.tensors,
            "ops": self.ops,
            "input": "input", "output": "logits",
            "exps": self.exps, "scales": self.scales,
            "fusion": self.fusion,
        }


def quantize(cfg: dict, weights: dict, calib: dict, out_dir: Path | None, fusion: bool):
    """Quantize float `weights` with calibration `calib`.  With `out_dir`, writes
    qgraph.json + qweights.bin there and returns the qgraph dict; without, returns
    (qgraph dict, blob bytes)."""
    if out_dir is not None:
        out_dir = Path(out_dir)
        out_dir.mkdir(parents=True, exist_ok=True)
        blob = TensorBlob(out_dir / "qweights.bin")
    else:
        blob = TensorBlob()
    try:
        g = Quantizer(cfg, weights, calib, fusion, blob).run()
    finally:
        blob.close()
    if out_dir is None:
        return g, blob.bytes()
    (out_dir / "qgraph.json").write_text(json.dumps(g, indent=1))
    return g


# ---------------------------------------------------------------------------------------
# Random-init float model and its calibration forward pass
# ---------------------------------------------------------------------------------------
def init_weights(cfg: ArchConfig, seed: int, device: str = "cpu") -> dict:
    """Float32 weights named like the reference exporter (export.py role names)."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def normal(*shape, std=0.02):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std

    W = {"embed": normal(cfg.vocab, cfg.dim)}
    qd, kvd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    for i in range(cfg.n_layers):
        p = f"l{i}"
        W[f"{p}_attn_norm"] = torch.ones(cfg.dim, device=device)
        W[f"{p}_wq"] = normal(qd, cfg.dim)
        W[f"{p}_wk"] = normal(kvd, cfg.dim)
        W[f"{p}_wv"] = normal(kvd, cfg.dim)
        if cfg.qkv_bias:
            W[f"{p}_bq"] = normal(qd, std=cfg.bias_std) if cfg.bias_std else torch.zeros(qd, device=device)
            W[f"{p}_bk"] = normal(kvd, std=cfg.bias_std) if cfg.bias_std else torch.zeros(kvd, device=device)
            W[f"{p}_bv"] = normal(kvd, std=cfg.bias_std) if cfg.bias_std else torch.zeros(kvd, device=device)
        if cfg.qk_norm:
            W[f"{p}_q_norm"] = torch.ones(cfg.head_dim, device=device)
            W[f"{p}_k_norm"] = torch.ones(cfg.head_dim, device=device)
        W[f"{p}_wo"] = normal(cfg.dim, qd)
        W[f"{p}_ffn_norm"] = torch.ones(cfg.dim, device=device)
        W[f"{p}_wg"] = normal(cfg.ffn, cfg.dim)
        W[f"{p}_wu"] = normal(cfg.ffn, cfg.dim)
        W[f"{p}_wd"] = normal(cfg.dim, cfg.ffn)
    W["norm"] = torch.ones(cfg.dim, device=device)
    W["lm_head"] = W["embed"] if cfg.tied else normal(cfg.vocab, cfg.dim)
    return W


def float_forward(cfg: ArchConfig, W: dict, ids: list[int], device: str = "cpu", rec=None, rec_rms=None):
    """Float32 forward of the architecture over one token sequence (causal, one pass);
    returns logits [T][vocab].  `rec(name, t)` / `rec_rms(name, t, width)` observe the named
    activations (the calibration hooks of calibrate.py:95-133)."""
    import torch
    import torch.nn.functional as F

    rec = rec or (lambda name, t: None)
    rec_rms = rec_rms or (lambda name, t, width: None)
    H, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

    def norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * w

    inv = cfg.rope_base ** (-torch.arange(0, D, 2, dtype=torch.float32, device=device) / D)
    with torch.no_grad():
        T = len(ids)
        tok = torch.tensor(ids, dtype=torch.long, device=device)
        ang = torch.outer(torch.arange(T, dtype=torch.float32, device=device), inv)
        ang = torch.cat((ang, ang), dim=-1)
        cos, sin = ang.cos(), ang.sin()

        def rot(x):  # x [H, T, D]
            half = D // 2
            return x * cos + torch.cat((-x[..., half:], x[..., :half]), -1) * sin

        x = W["embed"][tok]
        rec("input", x)
        resid = "input"
        for i in range(cfg.n_layers):
            p = f"l{i}"
            rec_rms(resid, x, cfg.dim)
            h = norm(x, W[f"{p}_attn_norm"])
            rec(f"{p}.h", h)
            q = h @ W[f"{p}_wq"].T
            k = h @ W[f"{p}_wk"].T
            v = h @ W[f"{p}_wv"].T
            if cfg.qkv_bias:
                q, k, v = q + W[f"{p}_bq"], k + W[f"{p}_bk"], v + W[f"{p}_bv"]
            rec(f"{p}.q", q)
            rec(f"{p}.k", k)
            rec(f"{p}.v", v)
            q = q.view(T, H, D)
            k = k.view(T, Hkv, D)
            if cfg.qk_norm:
                rec_rms(f"{p}.q", q, D)
                rec_rms(f"{p}.k", k, D)
                q = norm(q, W[f"{p}_q_norm"])
                k = norm(k, W[f"{p}_k_norm"])
                rec(f"{p}.qn", q)
                rec(f"{p}.kn", k)
            qr = rot(q.transpose(0, 1))
            kr = rot(k.transpose(0, 1))
            rec(f"{p}.qr", qr)
            rec(f"{p}.kr", kr)
            vv = v.view(T, Hkv, D).transpose(0, 1)
            rep = H // Hkv
            a = F.scaled_dot_product_attention(qr[None], kr.repeat_interleave(rep, 0)[None],
                                               vv.repeat_interleave(rep, 0)[None], is_causal=True)[0]
            a = a.transpose(0, 1).reshape(T, H * D)
            rec(f"{p}.a", a)
            o = a @ W[f"{p}_wo"].T
            rec(f"{p}.o", o)
            x1 = x + o
            rec(f"{p}.x1", x1)
            rec_rms(f"{p}.x1", x1, cfg.dim)
            h2 = norm(x1, W[f"{p}_ffn_norm"])
            rec(f"{p}.h2", h2)
            g = h2 @ W[f"{p}_wg"].T
            u = h2 @ W[f"{p}_wu"].T
            rec(f"{p}.g", g)
            rec(f"{p}.u", u)
            sg = F.silu(g)
            rec(f"{p}.sg", sg)
            f = sg * u
            rec(f"{p}.f", f)
            d = f @ W[f"{p}_wd"].T
            rec(f"{p}.d", d)
            x = x1 + d
            rec(f"{p}.x2", x)
            resid = f"{p}.x2"
        rec_rms(resid, x, cfg.dim)
        hn = norm(x, W["norm"])
        rec("hn", hn)
        logits = hn @ W["lm_head"].T
        rec("logits", logits)
        return logits


def calibrate(cfg: ArchConfig, W: dict, sequences: list[list[int]], device: str = "cpu") -> dict:
    """Abs-max of every named activation and RMS minimum of every RMSNorm input over
    `sequences`, from a float32 forward pass of the architecture (calibrate.py:95-133)."""
    absmax: dict[str, float] = {}
    rms_min: dict[str, float] = {}

    def rec(name, t):
        v = float(t.abs().max())
        if not math.isfinite(v):
            raise ValueError(f"nonfinite calibration activation {name!r}")
        absmax[name] = max(absmax.get(name, 0.0), v)

    def rec_rms(name, t, width):
        r = float(t.double().reshape(-1, width).square().mean(-1).sqrt().min())
        rms_min[name] = min(rms_min.get(name, float("inf")), r)

    for ids in sequences:
        float_forward(cfg, W, ids, device, rec, rec_rms)
    return absmax | {k + ".rms_min": v for k, v in rms_min.items()}


def build_qgraph(cfg: ArchConfig, out_dir, *, seed: int = 0, fusion: bool = True, calib_seqs: int = 4,
                 calib_len: int = 64, device: str = "cpu") -> dict:
    """Random-init `cfg`, calibrate, quantize, write out_dir/{qgraph.json, qweights.bin,
    manifest.json}.  Deterministic for a given (cfg, seed, device)."""
    out_dir = Path(out_dir)
    W = init_weights(cfg, seed, device)
    rng = np.random.default_rng(seed)
    L = min(calib_len, cfg.max_seq)
    seqs = [rng.integers(0, cfg.vocab, L).tolist() for _ in range(calib_seqs)]
    calib = calibrate(cfg, W, seqs, device)
    qcfg = {"dim": cfg.dim, "n_layers": cfg.n_layers, "n_heads": cfg.n_heads, "n_kv_heads": cfg.n_kv_heads,
            "head_dim": cfg.head_dim, "ffn": cfg.ffn, "vocab": cfg.vocab, "max_seq": cfg.max_seq,
            "rope_base": cfg.rope_base, "rms_eps": cfg.rms_eps}
    g = quantize(qcfg, W, calib, out_dir, fusion)
    (out_dir / "calib.json").write_text(json.dumps(calib, indent=1))
    (out_dir / "manifest.json").write_text(json.dumps({"arch": cfg.to_dict(), "seed": seed, "fusion": fusion,
                                                       "calib_seqs": calib_seqs, "calib_len": L,
                                                       "device": device}, indent=1))
    return g


def ensure_artefact(name: str, root, *, seed: int = 0, fusion: bool = True, device: str = "cpu") -> Path:
    """Path of the artefact for config `name` under `root`, generating it if absent."""
    cfg = CONFIGS[name]
    d = Path(root) / f"{name}_s{seed}_{'v2' if fusion else 'v1'}"
    if (d / "qgraph.json").exists() and (d / "manifest.json").exists():
        return d
    build_qgraph(cfg, d, seed=seed, fusion=fusion, device=device)
    return d
