"""GPU parity at the benchmark configs' real shapes: every config's dimensions, batch and
context (only the layer count is cut to 2, so the oracle finishes in seconds per sequence
and the artefact stays small).  The launch shapes that decide correctness at scale are the
ones the bench runs: tensor-core tile and split-K choices at the full N and K, decode
attention cluster sizes for the full number of (sequence, KV head) units and key slices of
the full context (C4: 4224 positions, 16 tiles of 256 keys), the wide-row RMSNorm at
dim 4096, the persistent vocabulary projection at vocab 151936 / 128256, and the B = 1
GEMV path.

Per config, for the chosen sequences of the batch, against the CPU oracle (bit for bit):
  * the record of every prefill chunk (argmax of its last valid row);
  * the tokens of the device-resident decode loop (CUDA graph, argmax-only output);
  * the logits rows and argmax of host-driven decode launches through the C ABI;
  * every named activation of a decode launch (a session that keeps activations).
"""
from __future__ import annotations

import dataclasses
import math
import os
from pathlib import Path

import numpy as np
import pytest

from oracle import golden_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from llaccel_b200 import artefacts as A  # noqa: E402
from llaccel_b200 import build as _build  # noqa: E402

_build.build()
from llaccel_b200.cuda_backend import CudaModel  # noqa: E402

N_DEC = 3
LAYERS = 2
# case: (config, sequences per launch, prompt tokens, sequences checked against the oracle)
CASES = {
    "c2": ("c2", 32, 128, (0, 31)),
    "c2_b1": ("c2", 1, 128, (0,)),
    "c3": ("c3", 128, 512, (0, 127)),
    "c4": ("c4", 64, 4096, (63,)),
    "c5": ("c5", 256, 1024, (0, 255)),
    "c5_b1": ("c5", 1, 1024, (0,)),
}

_ORACLE_CACHE: dict = {}


@pytest.fixture(scope="module")
def art_root(tmp_path_factory) -> Path:
    root = os.environ.get("LLX_TEST_ARTEFACTS")
    return Path(root) if root else tmp_path_factory.mktemp("config_scale")


def _artefact(config: str, root: Path):
    cfg = dataclasses.replace(A.CONFIGS[config], name=f"{config}_l{LAYERS}", n_layers=LAYERS)
    d = root / f"{cfg.name}_s0_v2"
    if not (d / "manifest.json").exists():
        A.build_qgraph(cfg, d, seed=0, fusion=True, device="cuda")
    return d, cfg


def _prompts(vocab: int, B: int, P: int) -> np.ndarray:
    # the same generator for every batch size: sequence b's prompt does not depend on B
    return np.random.default_rng(1000).integers(0, vocab, (max(B, 256), P)).astype(np.int32)[:B]


def _oracle(d: Path, prompt: list[int]) -> dict:
    """The golden model's prefill records, N_DEC decode launches (logits and argmax) and the
    named activations of the first decode launch, for one sequence."""
    key = (str(d), tuple(prompt))
    if key in _ORACLE_CACHE:
        return _ORACLE_CACHE[key]
    o = O.OracleModel(d)
    rows = o.prefill(prompt)
    L, pm, V = len(prompt), o.prefill_m, o.vocab
    pre_am = [int(np.argmax(rows[min(L, (c + 1) * pm) - 1][:V])) for c in range(math.ceil(L / pm))]
    nxt = pre_am[-1]
    dec_logits, dec_am, acts = [], [], []
    for i in range(N_DEC):
        lg = o.decode(nxt, L + i, acts if i == 0 else None)
        dec_logits.append(np.asarray(lg, np.int64))
        nxt = int(np.argmax(lg[:V]))
        dec_am.append(nxt)
    out = {"prefill_am": pre_am, "dec_logits": dec_logits, "dec_am": dec_am, "acts0": acts[0]["acts"]}
    _ORACLE_CACHE[key] = out
    return out


@pytest.mark.parametrize("case", list(CASES))
def test_config_scale_matches_oracle(art_root, case):
    config, B, P, seqs = CASES[case]
    d, cfg = _artefact(config, art_root)
    prompts = _prompts(cfg.vocab, B, P)
    want = {b: _oracle(d, prompts[b].tolist()) for b in seqs}
    n_chunks = math.ceil(P / 16)

    # ---- production session (the bench's launch sizes) ----
    max_rows = max(16, min(P, 512, (65536 // B) // 16 * 16))
    with CudaModel(d, batch=B, max_rows=max_rows) as m:
        recs = m.generate_batch(prompts.tolist(), 0, with_logits=False)
        for b in seqs:
            assert recs[b]["argmax_per_step"][:n_chunks] == want[b]["prefill_am"], f"{case}: prefill records, seq {b}"
        first = np.array([r["argmax_per_step"][-1] for r in recs], np.int32)
        # device-resident decode loop: argmax-only graph, tokens fed back on the device
        m.set_tokens(first)
        m.decode_async(P, N_DEC)
        m.sync()
        hist = m.history(N_DEC)
        for b in seqs:
            assert hist[:, b].tolist() == want[b]["dec_am"], f"{case}: device decode loop tokens, seq {b}"
        # host-driven launches through the C ABI with the logits rows
        cur = first.copy()
        for i in range(N_DEC):
            lg = m._launch_tokens(cur.reshape(B, 1), 1, P + i, None)[:, 0]
            for b in seqs:
                np.testing.assert_array_equal(lg[b], want[b]["dec_logits"][i], err_msg=f"{case}: decode {i} logits, seq {b}")
            cur = np.argmax(lg[:, : cfg.vocab], axis=1).astype(np.int32)
            assert cur.tolist() == hist[i].tolist(), f"{case}: host loop vs device loop, decode {i}"

    # ---- every named activation of the first decode launch (activations kept) ----
    with CudaModel(d, batch=B, max_rows=64, keep_acts=True) as m:
        recs = m.generate_batch(prompts.tolist(), 0, prefill_rows=64 if P >= 64 else 0, with_logits=False)
        for b in seqs:
            assert recs[b]["argmax_per_step"][:n_chunks] == want[b]["prefill_am"], f"{case}: prefill records (kept), seq {b}"
        acts: dict = {}
        m._launch_tokens(first.reshape(B, 1), 1, P, acts)
        for b in seqs:
            ref = want[b]["acts0"]
            missing = sorted(set(ref) - set(acts))
            assert not missing, f"{case}: activations not produced: {missing[:5]}"
            for name, arr in ref.items():
                np.testing.assert_array_equal(acts[name][b], np.asarray(arr)[0], err_msg=f"{case}: {name}, seq {b}")
