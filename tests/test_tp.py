"""Tensor-parallel sharding (llaccel_b200.tp) checked on the CPU oracle.

The ranks' graphs, run in lockstep with an exact int32 all-reduce, must reproduce the
reference's golden records of the unsharded graph bit for bit (logits of every recorded
row, argmax, generated tokens), for the reference-made fixtures and generator graphs."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from llaccel_b200 import tp
from oracle.golden_oracle import OracleModel
from oracle.tp_oracle import TPOracle


def _shard_all(src, tmp_path, world):
    return [tp.shard(src, tmp_path / f"r{r}", r, world) and tmp_path / f"r{r}" for r in range(world)]


@pytest.mark.parametrize("name", ["c1_v2", "c1_v1", "qwen3_tiny", "d128_tiny"])
def test_tp2_generate_matches_golden(tmp_path, name):
    src = GOLDEN / name
    dirs = _shard_all(src, tmp_path, 2)
    rec = json.loads((src / "golden.json").read_text())
    got = TPOracle(dirs).generate(rec["prompt_tokens"], len(rec["generated"]))
    assert got == rec


def test_tp_shard_geometry(tmp_path):
    src = GOLDEN / "c1_v2"
    g = json.loads((src / "qgraph.json").read_text())
    world = 2
    r1 = tp.shard(src, tmp_path / "r1", 1, world)
    md = r1["model"]
    assert md["n_heads"] == g["model"]["n_heads"] // world
    assert md["n_kv_heads"] == g["model"]["n_kv_heads"] // world
    assert md["vocab_padded"] == g["model"]["vocab_padded"] // world
    assert md["tp"] == {"rank": 1, "world": 2, "vocab_offset": g["model"]["vocab_padded"] // 2,
                        "vocab_padded_full": g["model"]["vocab_padded"]}
    kinds = [o["op"] for o in r1["ops"]]
    # two row-split linears per layer (o, down), each partial -> all-reduce -> requant
    n_layers = g["model"]["n_layers"]
    assert kinds.count("linear_partial") == 2 * n_layers
    assert kinds.count("allreduce") == 2 * n_layers
    assert kinds.count("requant") == 2 * n_layers
    for i, k in enumerate(kinds):
        if k == "linear_partial":
            assert kinds[i + 1] == "allreduce" and kinds[i + 2] == "requant"
    # the row-split weights hold this rank's K columns
    T, T1 = g["tensors"], r1["tensors"]
    assert T1["l0_wo"]["shape"] == [T["l0_wo"]["shape"][0], T["l0_wo"]["shape"][1] // world]
    assert T1["l0_wq"]["shape"] == [T["l0_wq"]["shape"][0] // world, T["l0_wq"]["shape"][1]]
    blob = np.fromfile(src / "qweights.bin", dtype=np.uint8)
    blob1 = np.fromfile(tmp_path / "r1" / "qweights.bin", dtype=np.uint8)
    wo = np.frombuffer(blob, "<i1", int(np.prod(T["l0_wo"]["shape"])), T["l0_wo"]["offset"]).reshape(T["l0_wo"]["shape"])
    wo1 = np.frombuffer(blob1, "<i1", int(np.prod(T1["l0_wo"]["shape"])), T1["l0_wo"]["offset"]).reshape(T1["l0_wo"]["shape"])
    k = T["l0_wo"]["shape"][1] // world
    np.testing.assert_array_equal(wo1, wo[:, k:])


def test_tp_world1_is_identity(tmp_path):
    src = GOLDEN / "qwen3_tiny"
    tp.shard(src, tmp_path / "r0", 0, 1)
    rec = json.loads((src / "golden.json").read_text())
    got = TPOracle([tmp_path / "r0"]).generate(rec["prompt_tokens"], len(rec["generated"]))
    assert got == rec


def test_tp_chunked_launches_match_unsharded(tmp_path):
    """Chunked launches of the sharded graph give the unsharded logits row for row."""
    src = GOLDEN / "c1_v2"
    dirs = _shard_all(src, tmp_path, 2)
    ref, tpm = OracleModel(src), TPOracle(dirs)
    rng = np.random.default_rng(7)
    toks = rng.integers(0, ref.vocab, 20).tolist()
    ref.reset()
    tpm.reset()
    for start in range(0, 20, 5):
        rows = ref.embed_rows(toks[start:start + 5], 5)
        np.testing.assert_array_equal(tpm.run_chunk(rows, start), ref.run_chunk(rows, start))


def test_tp_rejects_indivisible_heads(tmp_path):
    with pytest.raises(ValueError, match="split"):
        tp.shard(GOLDEN / "qwen2_tiny", tmp_path / "r0", 0, 2)  # one KV head
    with pytest.raises(ValueError):
        tp.shard(GOLDEN / "c1_v2", tmp_path / "r0", 2, 2)


def test_tp4_generator_graph(tmp_path):
    """World 4 on a generator graph with 4 KV heads (the C5 layout at a toy size)."""
    from llaccel_b200 import artefacts as A
    cfg = A.ArchConfig("tp4_tiny", 128, 2, 8, 4, 32, 256, 250, 64, 1e4, 1e-5)
    src = tmp_path / "full"
    A.build_qgraph(cfg, src, seed=3, fusion=True, device="cpu")
    dirs = _shard_all(src, tmp_path, 4)
    ref = OracleModel(src)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 21).tolist()
    want = ref.generate(prompt, 12)
    got = TPOracle(dirs).generate(prompt, 12)
    assert got == want
    assert len(set(want["generated"])) > 1  # not a degenerate constant stream
