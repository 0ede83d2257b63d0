"""Tensor-parallel CPU oracle -- TEST INFRASTRUCTURE ONLY.

Runs the rank-local graphs of one tensor-parallel group (written by
`llaccel_b200.tp.shard`) in lockstep on the CPU: every rank executes op i before any rank
executes op i+1, and an `allreduce` op replaces each rank's int32 partial accumulator by
the sum over ranks (the exact integer sum an NCCL int32 all-reduce computes).  The logits
of a launch are the ranks' vocabulary shards concatenated in rank order, so `generate`
returns the same golden.json record as the unsharded `OracleModel.generate`
(golden.py:399-440), which is what the tests compare.

The reference has no tensor parallelism; this runner only restates its single-device
algorithm over split weights, so its records must equal the unsharded golden records.
"""
from __future__ import annotations

import numpy as np

from .golden_oracle import OracleModel


class TPOracle(OracleModel):
    """OracleModel over the rank graphs `dirs` (rank order)."""

    def __init__(self, dirs) -> None:
        self.ranks = [OracleModel(d) for d in dirs]
        super().__init__(dirs[0])
        tp = self.q.model.get("tp")
        if not tp or tp["world"] != len(dirs):
            raise ValueError("rank graphs do not form one tensor-parallel group")
        for r, m in enumerate(self.ranks):
            t = m.q.model["tp"]
            if t["rank"] != r or len(m.q.ops) != len(self.q.ops):
                raise ValueError(f"rank {r}: graph does not belong to this group")
        self.vocab_padded = int(tp["vocab_padded_full"])

    def reset(self) -> None:
        for m in getattr(self, "ranks", []):
            m.reset()

    def run_chunk(self, rows, pos, acts=None):
        rows = np.asarray(rows, dtype=np.int64)
        M = rows.shape[0]
        if pos < 0 or pos + M > self.max_seq:
            raise ValueError(f"positions {pos}..{pos + M - 1} exceed max_seq={self.max_seq}")
        act = [{m.q.input_name: rows} for m in self.ranks]
        for i in range(len(self.q.ops)):
            ops = [m.q.ops[i] for m in self.ranks]
            if ops[0]["op"] == "allreduce":
                total = sum(a[ops[0]["in"]] for a in act)
                if np.abs(total).max(initial=0) >= 2**31:
                    raise ValueError("int32 all-reduce overflow")
                for a, op in zip(act, ops):
                    a[op["out"]] = total
            else:
                for m, a, op in zip(self.ranks, act, ops):
                    m.step(op, a, pos)
        if acts is not None:
            acts.update(act[0])
        out = self.q.output_name
        return np.concatenate([a[out] for a in act], axis=1)
