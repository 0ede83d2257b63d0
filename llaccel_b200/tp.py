"""Tensor-parallel sharding of a quantized graph: qgraph dir -> one rank-local qgraph dir.

The integer datapath splits exactly:

* a linear whose input is replicated is split by output channels ("column parallel"):
  q / k / v by attention heads, gate / up by FFN channels, lm_head by vocabulary.  Its
  rank computes its channels with the unchanged per-channel requant, bias and epilogue;
* a linear whose input is split (o by heads, down by FFN channels) is split by K ("row
  parallel"): each rank produces int32 partial sums (op `linear_partial`), an `allreduce`
  (int32 sum, exact: integer addition is associative and |sum| < 2^31) restores the full
  accumulator, and a `requant` op applies bias, requant and epilogue once, replicated.
  Reduce-then-requant is the only exact order because requant is nonlinear;
* RMSNorm, embedding and residual adds run replicated on full rows; RoPE, KV writes and
  attention run on the rank's heads (query heads r*H/g.., KV heads r*Hkv/g..);
* the logits stay split by vocabulary; the argmax is the max over ranks of the packed key
  (logit, lowest global index), an exact all-reduce (model.tp.vocab_offset).

Every other op is elementwise and follows its input's split.  The transform only slices
tensors and rewrites the op list; tests/test_tp.py checks on the CPU oracle that the ranks'
graphs, with the all-reduce summed across ranks, reproduce the unsharded golden bit for bit.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

_NP = {"i8": "<i1", "i16": "<i2", "i32": "<i4", "rq": "<i4"}


class _Blob:
    def __init__(self, path: Path) -> None:
        self.fh = open(path, "wb")
        self.off = 0
        self.tensors: dict[str, dict] = {}

    def add(self, name: str, arr: np.ndarray, dtype: str, exp=None) -> None:
        raw = np.ascontiguousarray(arr.astype(_NP[dtype])).tobytes()
        shape = list(arr.shape[:-1]) if dtype == "rq" else list(arr.shape)
        spec = {"dtype": dtype, "shape": [int(s) for s in shape], "offset": self.off}
        if exp is not None:
            spec["exp"] = exp
        self.tensors[name] = spec
        pad = (-len(raw)) % 64
        self.fh.write(raw + b"\0" * pad)
        self.off += len(raw) + pad

    def close(self) -> None:
        self.fh.close()


def _tensor(blob, spec):
    n = int(np.prod(spec["shape"]))
    if spec["dtype"] == "rq":
        return np.frombuffer(blob, dtype="<i4", count=2 * n, offset=spec["offset"]).reshape(n, 2)
    return np.frombuffer(blob, dtype=_NP[spec["dtype"]], count=n, offset=spec["offset"]).reshape(spec["shape"])


def shard(src, dst, rank: int, world: int) -> dict:
    """Write the rank-local qgraph of `src` for `rank` of `world` into `dst`; returns it."""
    src, dst = Path(src), Path(dst)
    g = json.loads((src / "qgraph.json").read_text())
    blob = np.memmap(src / g.get("weights_file", "qweights.bin"), dtype=np.uint8, mode="r")
    T = g["tensors"]
    md = dict(g["model"])
    H, Hkv = int(md["n_heads"]), int(md["n_kv_heads"])
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if H % world or Hkv % world:
        raise ValueError(f"heads {H}/{Hkv} do not split over {world} ranks")
    dst.mkdir(parents=True, exist_ok=True)
    out = _Blob(dst / "qweights.bin")
    added: set[str] = set()

    def copy(name):
        if name in added or name is None:
            return
        spec = T[name]
        out.add(name, np.array(_tensor(blob, spec)), spec["dtype"], spec.get("exp"))
        added.add(name)

    # split state of every activation: None = full, else (c0, c1) of the full channel range
    split: dict[str, tuple[int, int] | None] = {g.get("input", "input"): None}
    cols: dict[str, int] = {g.get("input", "input"): int(md["dim"])}
    ops = []
    for tname in ("embed", "rope_cos", "rope_sin"):
        copy(tname)

    def part(n):  # this rank's range of n channels
        if n % world:
            raise ValueError(f"{n} channels do not split over {world} ranks")
        k = n // world
        return rank * k, (rank + 1) * k

    for op in g["ops"]:
        k = op["op"]
        if k == "linear":
            N, K = int(op["N"]), int(op["K"])
            W = _tensor(blob, T[op["w"]])
            rq = _tensor(blob, T[op["rq"]])
            bias = _tensor(blob, T[op["bias"]]) if op.get("bias") else None
            if split[op["in"]] is None:
                c0, c1 = part(N)
                out.add(op["w"], np.array(W[c0:c1]), "i8")
                out.add(op["rq"], np.array(rq[c0:c1]), "rq")
                if bias is not None:
                    out.add(op["bias"], np.array(bias[c0:c1]), "i32")
                no = dict(op, N=c1 - c0)
                if op.get("epilogue", "none") in ("resadd", "mul") and split[op["aux"]] != (c0, c1):
                    raise ValueError(f"linear {op['out']}: epilogue operand is not split like its output")
                ops.append(no)
                split[op["out"]], cols[op["out"]] = (c0, c1), c1 - c0
            else:
                k0, k1 = split[op["in"]]
                if k1 - k0 != cols[op["in"]] or K != (k1 - k0) * world:
                    raise ValueError(f"linear {op['out']}: input split does not match K")
                acc = op["out"] + ".acc"
                out.add(op["w"], np.ascontiguousarray(W[:, k0:k1]), "i8")
                ops.append({"op": "linear_partial", "in": op["in"], "w": op["w"], "out": acc, "N": N, "K": k1 - k0})
                ops.append({"op": "allreduce", "in": acc, "out": acc, "reduce": "sum"})
                copy(op["rq"])
                copy(op.get("bias"))
                rq_op = {"op": "requant", "in": acc, "rq": op["rq"], "bias": op.get("bias"), "out": op["out"], "N": N,
                         "out_dtype": op.get("out_dtype", "i16"), "epilogue": op.get("epilogue", "none"),
                         "aux": op.get("aux"), "aux_shift": op.get("aux_shift", 0), "silu": op.get("silu")}
                if rq_op["epilogue"] in ("resadd", "mul") and split[op["aux"]] is not None:
                    raise ValueError(f"linear {op['out']}: row-parallel epilogue needs a full operand")
                ops.append(rq_op)
                split[acc], cols[acc] = None, N
                split[op["out"]], cols[op["out"]] = None, N
        elif k == "rmsnorm":
            copy(op["gamma"])
            heads = int(op.get("heads", 1))
            if split[op["in"]] is not None:
                if heads == 1:
                    raise ValueError(f"rmsnorm {op['out']}: full-row norm of a split activation")
                no = dict(op, heads=heads // world)
            else:
                no = dict(op)
            ops.append(no)
            split[op["out"]], cols[op["out"]] = split[op["in"]], cols[op["in"]]
        elif k == "rope":
            h = int(op["H"])
            no = dict(op, H=h // world) if split[op["in"]] is not None else dict(op)
            ops.append(no)
            split[op["out"]], cols[op["out"]] = split[op["in"]], cols[op["in"]]
        elif k == "kv_write":
            if split[op["k"]] is None or split[op["v"]] is None:
                raise ValueError("kv_write of a replicated key/value")
            ops.append(dict(op, Hkv=int(op["Hkv"]) // world))
        elif k == "attention":
            if split[op["q"]] is None:
                raise ValueError("attention over replicated queries")
            ops.append(dict(op, H=int(op["H"]) // world, Hkv=int(op["Hkv"]) // world))
            split[op["out"]], cols[op["out"]] = split[op["q"]], cols[op["q"]]
        elif k in ("quant", "silu"):
            ops.append(dict(op))
            split[op["out"]], cols[op["out"]] = split[op["in"]], cols[op["in"]]
        elif k in ("add", "mul"):
            if split[op["a"]] != split[op["b"]]:
                raise ValueError(f"{k} {op['out']}: operands split differently")
            ops.append(dict(op))
            split[op["out"]], cols[op["out"]] = split[op["a"]], cols[op["a"]]
        else:
            raise ValueError(f"unknown qgraph op {k!r}")
    out.close()
    out_name = g.get("output", "logits")
    vsplit = split[out_name]
    if vsplit is None:
        raise ValueError("the output must be split by vocabulary")
    tp = {"rank": rank, "world": world, "vocab_offset": vsplit[0], "vocab_padded_full": int(md["vocab_padded"])}
    md["vocab_padded"] = vsplit[1] - vsplit[0]
    md["n_heads"], md["n_kv_heads"] = H // world, Hkv // world
    # argmax over global channels < vocab: this rank's shard holds channels [c0, c1)
    md["tp"] = tp
    rg = {"model": md, "weights_file": "qweights.bin", "tensors": out.tensors, "ops": ops,
          "input": g.get("input", "input"), "output": out_name}
    (dst / "qgraph.json").write_text(json.dumps(rg, indent=1))
    return rg
