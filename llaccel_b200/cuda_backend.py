"""`CudaModel`: the golden model's interface (python/llaccel/golden.py:246-440) on the B200
backend, through the C ABI in include/llx.h (llaccel_b200/_lib/libllx.so).

Same constructor argument (a qgraph directory), same methods (`reset`, `run_chunk`,
`prefill`, `decode`, `generate`), same return values (int64 numpy logits, the golden.json
record dict) and the same ValueError messages for bad positions, empty prompts and
oversized requests.  Extra: `batch` independent sequences per launch and
`generate_batch`, which runs whole-prompt prefill launches and a device-resident decode
loop and still returns one golden.json record per sequence.

There is no CPU fallback: constructing a CudaModel without the built library or a CUDA
device raises.
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libllx.so"

LLX_OK, LLX_ERR_INVALID, LLX_ERR_IO, LLX_ERR_CUDA, LLX_ERR_OOM, LLX_ERR_RANGE, LLX_ERR_UNSUPPORTED, LLX_ERR_DEVICE = range(8)

# exported symbols, with (restype, argtypes); tests check the library exports each of them
_I32P = C.POINTER(C.c_int32)
_I16P = C.POINTER(C.c_int16)
SIGNATURES = {
    "llx_model_load": (C.c_int, [C.c_char_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "llx_model_destroy": (None, [C.c_void_p]),
    "llx_model_get_info": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llx_session_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "llx_session_destroy": (None, [C.c_void_p]),
    "llx_session_reset": (C.c_int, [C.c_void_p]),
    "llx_run": (C.c_int, [C.c_void_p, _I32P, C.c_int, C.c_int, _I32P, C.c_int, _I16P, _I32P]),
    "llx_run_rows": (C.c_int, [C.c_void_p, _I16P, C.c_int, C.c_int, _I16P, _I32P]),
    "llx_generate": (C.c_int, [C.c_void_p, _I32P, C.c_int, C.c_int, C.c_int, _I32P, _I32P, _I16P,
                               C.POINTER(C.c_int)]),
    "llx_set_tokens": (C.c_int, [C.c_void_p, _I32P]),
    "llx_decode_async": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "llx_read_history": (C.c_int, [C.c_void_p, C.c_int, _I32P]),
    "llx_sync": (C.c_int, [C.c_void_p]),
    "llx_session_stream": (C.c_void_p, [C.c_void_p]),
    "llx_decode_launches_per_step": (C.c_int, [C.c_void_p]),
    "llx_plan_steps": (C.c_int, [C.c_void_p]),
    "llx_step_label": (C.c_char_p, [C.c_void_p, C.c_int]),
    "llx_profile_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_double),
                                     C.POINTER(C.c_double), C.c_int, C.POINTER(C.c_int)]),
    "llx_activation_count": (C.c_int, [C.c_void_p]),
    "llx_activation_name": (C.c_char_p, [C.c_void_p, C.c_int]),
    "llx_activation_shape": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "llx_read_activation": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    "llx_linear_argmax_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                            C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "llx_last_error": (C.c_char_p, []),
    "llx_version": (C.c_char_p, []),
    "llx_binary_version": (C.c_int, [C.c_int, C.c_void_p]),
    "llx_tp_unique_id": (C.c_int, [C.c_void_p]),
    "llx_tp_init": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
}


class LlxOpts(C.Structure):
    _fields_ = [("device", C.c_int), ("fuse", C.c_int), ("gemm_path", C.c_int), ("pdl", C.c_int)]


class LlxModelInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                                        "vocab_padded", "max_seq", "prefill_m", "E_RES", "E_LOGIT", "n_ops",
                                        "n_steps", "n_activations")] + [("weight_bytes", C.c_size_t)] + \
        [(n, C.c_int) for n in ("tp_world", "tp_rank", "vocab_base", "vocab_local")]


class LlxError(RuntimeError):
    def __init__(self, code: int, msg: str) -> None:
        super().__init__(msg)
        self.code = code


_lib_handle = None


def load_library(path: Path | str | None = None):
    """Load libllx.so (raises if it was not built: `python -m llaccel_b200.build`)."""
    global _lib_handle
    if _lib_handle is not None and path is None:
        return _lib_handle
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"CUDA backend library missing: {p} (build it with `python -m llaccel_b200.build`)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _lib_handle = lib
    return lib


def _check(lib, code: int) -> None:
    if code == LLX_OK:
        return
    msg = lib.llx_last_error().decode()
    if code in (LLX_ERR_INVALID, LLX_ERR_RANGE):
        raise ValueError(msg)
    raise LlxError(code, msg)


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for llx_tp_init; made on rank 0 and shared."""
    lib = load_library()
    buf = C.create_string_buffer(128)
    _check(lib, lib.llx_tp_unique_id(buf))
    return buf.raw


def _p32(a: np.ndarray):
    return a.ctypes.data_as(_I32P)


def _p16(a: np.ndarray):
    return a.ctypes.data_as(_I16P)


class CudaModel:
    """GoldenModel on the GPU.  `batch` sequences share each launch; `max_rows` bounds
    the rows per sequence of one launch (default: max_seq); `keep_acts` keeps every named
    activation of the last launch readable (needed for `acts=`)."""

    def __init__(self, qgraph_dir, *, batch: int = 1, device: int = 0, max_rows: int | None = None,
                 keep_acts: bool = False, fuse: bool = True, gemm_path: int = 0, pdl: bool = True,
                 share: "CudaModel | None" = None, tp: "tuple[int, int, bytes] | None" = None) -> None:
        """`share`: reuse the weights already loaded by another CudaModel (same device); this
        instance then owns only its session (KV cache, activations, stream).
        `tp`: (rank, world, unique_id) for a rank graph of a tensor-parallel group
        (llaccel_b200.tp.shard); every rank of the group constructs its model together and
        then makes the same calls in the same order."""
        self.lib = load_library()
        self.dir = Path(qgraph_dir)
        self.batch = int(batch)
        self._owns_model = share is None
        if share is not None:
            self._model = share._model
            self._shared_from = share  # keeps the owner alive
        else:
            opts = LlxOpts(int(device), 1 if fuse else 0, int(gemm_path), 1 if pdl else 0)
            self._model = C.c_void_p()
            _check(self.lib, self.lib.llx_model_load(str(self.dir).encode(), C.byref(opts), C.byref(self._model)))
            if tp is not None:
                rank, world, uid = tp
                uid_buf = C.create_string_buffer(bytes(uid), 128)
                code = self.lib.llx_tp_init(self._model, uid_buf, int(rank), int(world))
                if code != LLX_OK:
                    msg = self.lib.llx_last_error().decode()
                    self.lib.llx_model_destroy(self._model)
                    self._model = None
                    if code in (LLX_ERR_INVALID, LLX_ERR_RANGE):
                        raise ValueError(msg)
                    raise LlxError(code, msg)
        info = LlxModelInfo()
        _check(self.lib, self.lib.llx_model_get_info(self._model, C.byref(info)))
        self.info = info
        self.dim, self.n_layers, self.vocab = info.dim, info.n_layers, info.vocab
        self.vocab_padded, self.max_seq, self.prefill_m = info.vocab_padded, info.max_seq, info.prefill_m
        self.E_RES, self.E_LOGIT = info.E_RES, info.E_LOGIT
        self.max_rows = int(max_rows or self.max_seq)
        self.keep_acts = bool(keep_acts)
        self._sess = C.c_void_p()
        _check(self.lib, self.lib.llx_session_create(self._model, self.batch, self.max_rows, 1 if keep_acts else 0,
                                                     C.byref(self._sess)))
        self._embed = None
        self.act_names = [self.lib.llx_activation_name(self._model, i).decode()
                          for i in range(self.lib.llx_activation_count(self._model))]

    # ---- lifetime ---------------------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_sess", None):
            self.lib.llx_session_destroy(self._sess)
            self._sess = None
        if getattr(self, "_model", None):
            if getattr(self, "_owns_model", True):
                self.lib.llx_model_destroy(self._model)
            self._model = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- golden-model surface -----------------------------------------------------------------
    @property
    def embed(self) -> np.ndarray:
        """The i16 embedding table (host copy, read from the weight file)."""
        if self._embed is None:
            g = json.loads((self.dir / "qgraph.json").read_text())
            spec = g["tensors"]["embed"]
            blob = np.memmap(self.dir / g.get("weights_file", "qweights.bin"), dtype=np.uint8, mode="r")
            n = int(np.prod(spec["shape"]))
            self._embed = np.frombuffer(blob, dtype="<i2", count=n, offset=spec["offset"]).reshape(spec["shape"])
        return self._embed

    def reset(self) -> None:
        _check(self.lib, self.lib.llx_session_reset(self._sess))

    def embed_rows(self, tokens, M: int) -> np.ndarray:
        rows = np.zeros((M, self.dim), np.int64)
        for i, t in enumerate(tokens):
            rows[i] = self.embed[int(t)]
        return rows

    @staticmethod
    def argmax(logits_row: np.ndarray, vocab: int) -> int:
        return int(np.argmax(logits_row[:vocab]))

    def _read_acts(self) -> dict:
        out = {}
        for name in self.act_names:
            cols, elem = C.c_int(), C.c_int()
            _check(self.lib, self.lib.llx_activation_shape(self._model, name.encode(), C.byref(cols), C.byref(elem)))
            dt = np.int8 if elem.value == 1 else np.int16
            buf = np.empty(self.batch * self.max_rows * cols.value, dtype=dt)
            rows = C.c_int()
            _check(self.lib, self.lib.llx_read_activation(self._sess, name.encode(), buf.ctypes.data_as(C.c_void_p),
                                                          buf.nbytes, C.byref(rows)))
            out[name] = buf[: rows.value * cols.value].reshape(rows.value, cols.value).astype(np.int64)
        return out

    def run_chunk(self, rows, pos: int, acts: dict | None = None) -> np.ndarray:
        """rows [M][dim] (batch 1) or [batch][M][dim] i16 at E_RES -> logits [..][M][vocab_padded]."""
        r = np.asarray(rows)
        squeeze = r.ndim == 2
        if squeeze:
            r = r[None]
        if r.shape[0] != self.batch or r.shape[2] != self.dim:
            raise ValueError(f"rows must be [{self.batch}][M][{self.dim}]")
        M = r.shape[1]
        if pos < 0 or pos + M > self.max_seq:
            raise ValueError(f"positions {pos}..{pos + M - 1} exceed max_seq={self.max_seq}")
        if acts is not None and not self.keep_acts:
            raise ValueError("activation capture needs CudaModel(..., keep_acts=True)")
        r16 = np.ascontiguousarray(r, dtype=np.int16)
        logits = np.empty((self.batch, M, self.vocab_padded), np.int16)
        _check(self.lib, self.lib.llx_run_rows(self._sess, _p16(r16), M, int(pos), _p16(logits), None))
        if acts is not None:
            acts.update(self._read_acts())
        out = logits.astype(np.int64)
        return out[0] if squeeze else out

    def _launch_tokens(self, tokens: np.ndarray, M: int, pos: int, acts: dict | None):
        """tokens [batch][M] (-1 pad) -> logits [batch][M][vocab_padded] (int64)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.empty((self.batch, M, self.vocab_padded), np.int16)
        _check(self.lib, self.lib.llx_run(self._sess, _p32(t), M, int(pos), None, 0, _p16(logits), None))
        if acts is not None:
            acts.update(self._read_acts())
        return logits.astype(np.int64)

    def prefill(self, tokens, acts: list | None = None) -> list[np.ndarray]:
        """Chunked prefill (prefill_m rows per launch, zero pad rows) -- golden.py:379-390."""
        tokens = [int(t) for t in tokens]
        out = []
        for start in range(0, len(tokens), self.prefill_m):
            chunk = tokens[start : start + self.prefill_m]
            t = np.full((self.batch, self.prefill_m), -1, np.int32)
            t[:, : len(chunk)] = chunk
            a = {} if acts is not None else None
            logits = self._launch_tokens(t, self.prefill_m, start, a)[0]
            if acts is not None:
                acts.append({"kind": "prefill", "pos": start, "rows": self.prefill_m, "valid_rows": len(chunk), "acts": a})
            out.extend(logits[: len(chunk)])
        return out

    def decode(self, token: int, pos: int, acts: list | None = None) -> np.ndarray:
        a = {} if acts is not None else None
        t = np.full((self.batch, 1), int(token), np.int32)
        logits = self._launch_tokens(t, 1, pos, a)[0, 0]
        if acts is not None:
            acts.append({"kind": "decode", "pos": pos, "rows": 1, "valid_rows": 1, "acts": a})
        return logits

    def _record_meta(self) -> dict:
        return {"vocab": self.vocab, "vocab_padded": self.vocab_padded, "E_LOGIT": self.E_LOGIT, "E_RES": self.E_RES,
                "max_seq": self.max_seq}

    def _validate(self, prompt_tokens, n_tokens) -> list[int]:
        if not isinstance(n_tokens, int) or n_tokens < 0:
            raise ValueError("n_tokens must be a nonnegative integer")
        prompt = [int(t) for t in prompt_tokens]
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + n_tokens > self.max_seq:
            raise ValueError(f"prompt + tokens = {len(prompt) + n_tokens} exceeds max_seq={self.max_seq}")
        return prompt

    def generate(self, prompt_tokens, n_tokens: int, acts: list | None = None, *, fast: bool = True,
                 prefill_rows: int | None = None) -> dict:
        """Greedy generation; returns the golden.json record (golden.py:399-440).  With `acts`
        (or fast=False) the launches go one by one through llx_run exactly like the reference
        host loop; otherwise llx_generate runs whole-prompt prefill and the device decode loop."""
        prompt = self._validate(prompt_tokens, n_tokens)
        if acts is not None or not fast:
            return self._generate_host_loop(prompt, n_tokens, acts)
        if self.batch != 1:
            raise ValueError("generate() takes one sequence; use generate_batch for batch > 1")
        return self.generate_batch([prompt], n_tokens, prefill_rows=prefill_rows)[0]

    def _generate_host_loop(self, prompt, n_tokens, acts):
        if self.batch != 1:
            raise ValueError("the host-loop generate takes batch 1")
        self.reset()
        steps, argmaxes, rows_rec = [], [], []

        def record(kind, pos, valid, row):
            steps.append({"kind": kind, "pos": pos, "rows": self.prefill_m if kind == "prefill" else 1,
                          "valid_rows": valid})
            argmaxes.append(self.argmax(row, self.vocab))
            rows_rec.append([int(v) for v in row[: self.vocab]])
            return argmaxes[-1]

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
                "logits_last_rows": rows_rec, "steps": steps, "model": self._record_meta()}

    def generate_batch(self, prompts, n_tokens: int, *, prefill_rows: int | None = None,
                       with_logits: bool = True) -> list[dict]:
        """`batch` sequences of equal prompt length -> one golden.json record each.
        prefill_rows: rows per sequence per prefill launch (multiple of prefill_m; default
        the whole prompt, capped by max_rows); 0 mirrors the golden's prefill_m chunks."""
        P = [self._validate(p, n_tokens) for p in prompts]
        if len(P) != self.batch:
            raise ValueError(f"expected {self.batch} prompts")
        L = len(P[0])
        if any(len(p) != L for p in P):
            raise ValueError("generate_batch needs equal prompt lengths")
        if prefill_rows is None:
            pm = self.prefill_m
            prefill_rows = min(self.max_rows // pm * pm, math.ceil(L / pm) * pm)
        pr = np.ascontiguousarray(np.array(P, dtype=np.int32))
        n_chunks = math.ceil(L / self.prefill_m)
        n_launch_max = n_chunks + n_tokens
        gen = np.zeros((self.batch, max(n_tokens, 1)), np.int32)
        am = np.zeros((self.batch, n_launch_max), np.int32)
        lg = np.zeros((self.batch, n_launch_max, self.vocab), np.int16) if with_logits else None
        nl = C.c_int()
        _check(self.lib, self.lib.llx_generate(self._sess, _p32(pr), L, n_tokens, int(prefill_rows), _p32(gen),
                                               am.ctypes.data_as(_I32P),
                                               _p16(lg) if lg is not None else None, C.byref(nl)))
        n_launch = nl.value
        # the C side lays argmax/logits out as [batch][n_launch]; repack from the row stride used
        am = am.reshape(-1)[: self.batch * n_launch].reshape(self.batch, n_launch)
        if lg is not None:
            lg = lg.reshape(-1)[: self.batch * n_launch * self.vocab].reshape(self.batch, n_launch, self.vocab)
        recs = []
        for b in range(self.batch):
            steps = []
            for c in range(n_chunks):
                valid = min(L, (c + 1) * self.prefill_m) - c * self.prefill_m
                steps.append({"kind": "prefill", "pos": c * self.prefill_m, "rows": self.prefill_m, "valid_rows": valid})
            for i in range(n_launch - n_chunks):
                steps.append({"kind": "decode", "pos": L + i, "rows": 1, "valid_rows": 1})
            rec = {"prompt_tokens": P[b], "generated": gen[b, :n_tokens].tolist(),
                   "argmax_per_step": am[b].tolist(),
                   "logits_last_rows": lg[b].tolist() if lg is not None else None,
                   "steps": steps, "model": self._record_meta()}
            recs.append(rec)
        return recs

    # ---- device-resident decode (benchmark / serving) --------------------------------------
    def stream_handle(self) -> int:
        return int(self.lib.llx_session_stream(self._sess) or 0)

    def set_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(self.batch))
        _check(self.lib, self.lib.llx_set_tokens(self._sess, _p32(t)))

    def decode_async(self, pos: int, n_steps: int) -> None:
        _check(self.lib, self.lib.llx_decode_async(self._sess, int(pos), int(n_steps)))

    def sync(self) -> None:
        _check(self.lib, self.lib.llx_sync(self._sess))

    def history(self, n_steps: int) -> np.ndarray:
        h = np.zeros((n_steps, self.batch), np.int32)
        _check(self.lib, self.lib.llx_read_history(self._sess, int(n_steps), _p32(h)))
        return h

    def profile_decode(self, pos: int, iters: int = 20) -> list[dict]:
        """Per-kernel timing of the M=1 decode plan at `pos`: one dict per kernel with
        label, ms (average per launch), algorithmic bytes and ops."""
        n = self.lib.llx_plan_steps(self._model)
        ms = (C.c_float * n)()
        by = (C.c_double * n)()
        op = (C.c_double * n)()
        got = C.c_int()
        _check(self.lib, self.lib.llx_profile_decode(self._sess, int(pos), int(iters), ms, by, op, n, C.byref(got)))
        return [{"label": self.lib.llx_step_label(self._model, i).decode(), "ms": float(ms[i]), "bytes": float(by[i]),
                 "ops": float(op[i])} for i in range(got.value)]

    def decode_launches_per_step(self) -> int:
        n = self.lib.llx_decode_launches_per_step(self._sess)
        if n < 0:
            raise LlxError(LLX_ERR_CUDA, self.lib.llx_last_error().decode())
        return n


class CudaLanes:
    """`lanes` sessions over one loaded model, each holding batch/lanes of the sequences on
    its own CUDA stream.  Decode steps of different lanes are independent, so their kernel
    chains run concurrently and fill the GPU where one chain alone is latency-bound.
    Results are those of one session holding every sequence (sequences never interact)."""

    def __init__(self, qgraph_dir, *, batch: int, lanes: int, device: int = 0, max_rows: int | None = None,
                 **kw) -> None:
        if lanes < 1 or batch % lanes:
            raise ValueError("batch must be a multiple of lanes")
        self.batch, self.lanes, self.per = batch, lanes, batch // lanes
        first = CudaModel(qgraph_dir, batch=self.per, device=device, max_rows=max_rows, **kw)
        self.models = [first] + [CudaModel(qgraph_dir, batch=self.per, device=device, max_rows=max_rows, share=first)
                                 for _ in range(lanes - 1)]

    def generate_batch(self, prompts, n_tokens: int, **kw) -> list[dict]:
        out = []
        for i, m in enumerate(self.models):
            out.extend(m.generate_batch(prompts[i * self.per : (i + 1) * self.per], n_tokens, **kw))
        return out

    def set_tokens(self, tokens) -> None:
        t = np.asarray(tokens, dtype=np.int32).reshape(self.lanes, self.per)
        for m, tl in zip(self.models, t):
            m.set_tokens(tl)

    def decode_async(self, pos: int, n_steps: int) -> None:
        for m in self.models:
            m.decode_async(pos, n_steps)

    def sync(self) -> None:
        for m in self.models:
            m.sync()

    def history(self, n_steps: int) -> np.ndarray:
        return np.concatenate([m.history(n_steps) for m in self.models], axis=1)

    def streams(self) -> list[int]:
        return [m.stream_handle() for m in self.models]

    def close(self) -> None:
        for m in reversed(self.models):
            m.close()
