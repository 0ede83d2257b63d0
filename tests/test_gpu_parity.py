"""GPU parity: the CUDA backend (through the C ABI) against the reference's golden records
and against the CPU oracle, bit for bit.  Every comparison here is exact equality: the
datapath is integer-only, so there is no tolerance."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN, QGRAPH_FIXTURES
from oracle import golden_oracle as O
import qgraph_synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from llaccel_b200 import build as _build  # noqa: E402

_build.build()
from llaccel_b200.cuda_backend import CudaModel  # noqa: E402


def _rec(name):
    rec = json.loads((GOLDEN / name / "golden.json").read_text())
    return rec, rec["prompt_tokens"], len(rec["generated"])


@pytest.mark.parametrize("name", QGRAPH_FIXTURES)
def test_generate_matches_reference_record(name):
    rec, prompt, n = _rec(name)
    with CudaModel(GOLDEN / name) as m:
        assert m.generate(prompt, n) == rec


@pytest.mark.parametrize("name", QGRAPH_FIXTURES)
def test_host_loop_activations_match_reference(name):
    rec, prompt, n = _rec(name)
    want = np.load(GOLDEN / name / "acts.npz")
    acts: list = []
    with CudaModel(GOLDEN / name, keep_acts=True, max_rows=16) as m:
        got = m.generate(prompt, n, acts)
    assert got == rec
    for key in want.files:
        i, kind, pos, act = key.split("|", 3)
        st = acts[int(i)]
        assert st["kind"] == kind and st["pos"] == int(pos)
        np.testing.assert_array_equal(st["acts"][act].astype(np.int32), want[key], err_msg=key)


@pytest.mark.parametrize("name", ["fx_v1", "c1_v2", "qwen3_tiny", "d128_tiny"])
@pytest.mark.parametrize("fuse,gemm_path", [(False, 1), (False, 2), (False, 3), (False, 4), (True, 1), (True, 2),
                                             (True, 3), (True, 4)])
def test_plan_and_gemm_variants_are_identical(name, fuse, gemm_path):
    rec, prompt, n = _rec(name)
    with CudaModel(GOLDEN / name, fuse=fuse, gemm_path=gemm_path) as m:
        assert m.generate(prompt, n) == rec
        assert m.generate(prompt, n, fast=False) == rec


@pytest.mark.parametrize("name", ["c1_v2", "qwen2_tiny", "d128_tiny"])
def test_batch_matches_oracle_per_sequence(name):
    o = O.OracleModel(GOLDEN / name)
    rng = np.random.default_rng(7)
    B, L, n = 5, 21, 9
    prompts = rng.integers(0, o.vocab, (B, L)).tolist()
    with CudaModel(GOLDEN / name, batch=B) as m:
        for prefill_rows in (None, 0, 16):
            recs = m.generate_batch(prompts, n, prefill_rows=prefill_rows)
            for b in range(B):
                assert recs[b] == o.generate(prompts[b], n), (prefill_rows, b)


@pytest.mark.parametrize("cfg", [
    dict(seed=1),
    dict(seed=2, fuse=False),
    dict(seed=3, extreme=True),
    dict(seed=4, extreme=True, fuse=False, prob_bits=8),
    dict(seed=5, D=128, H=2, Hkv=1, dim=128, ffn=64, qk_norm=True),
    dict(seed=6, D=16, H=6, Hkv=3, dim=48, ffn=32, vocab=17, bias=False),
    dict(seed=7, D=64, H=4, Hkv=4, prefill_m=4, max_seq=48),
])
def test_stress_graphs_run_chunk_matches_oracle(tmp_path, cfg):
    d = qgraph_synth.build(tmp_path / "g", **cfg)
    o = O.OracleModel(d)
    rng = np.random.default_rng(cfg["seed"])
    with CudaModel(d, max_rows=16, keep_acts=True) as m:
        pos = 0
        for M in (16, 5, 1, 1, 9, 1):
            rows = o.embed[rng.integers(0, o.vocab, M)].astype(np.int64)
            rows[rng.random(M) < 0.2] = 0  # zero pad rows
            want_acts, got_acts = {}, {}
            want = o.run_chunk(rows, pos, want_acts)
            got = m.run_chunk(rows, pos, got_acts)
            np.testing.assert_array_equal(got, want)
            for k, v in want_acts.items():
                np.testing.assert_array_equal(got_acts[k], v, err_msg=f"{k} pos={pos} M={M}")
            pos += M


@pytest.mark.parametrize("K,N,epi,chain", [
    (64, 48, "none", 0), (128, 256, "none", 0), (896, 1152, "none", 0), (576, 576, "resadd", 0),
    (256, 4864, "silu", 0), (512, 512, "mul", 0), (4864, 64, "none", 0), (14336, 32, "none", 0),
    (352, 2048, "none", 96), (1024, 40000, "none", 0), (160, 8, "none", 0)])
@pytest.mark.parametrize("R", [1, 5, 16, 40, 128, 300])
def test_linear_paths_match_oracle(tmp_path, K, N, epi, chain, R):
    """Every GEMM schedule (GEMV, with several channel groups per block from N = 4736 at one
    row; tiled dp4a; tcgen05: the swapped-operand decode kernel for R <= 32 (path 3), the
    row-tile kernel with and without cluster split-K (path 4, and path 3 above 32 rows)) on
    full-range int8 operands against the oracle, for all four epilogues and i8 outputs."""
    d = qgraph_synth.build_linear(tmp_path / "lin", K=K, N=N, epi=epi, chain_i8=chain, seed=K + N + R)
    o = O.OracleModel(d)
    rng = np.random.default_rng(R)
    rows = rng.integers(-32768, 32768, (R, K))
    rows[0] = 32767
    rows[-1] = -32768
    want = o.run_chunk(rows, 0)
    for path in (3, 4, 1, 2):
        with CudaModel(d, max_rows=R, gemm_path=path) as m:
            np.testing.assert_array_equal(m.run_chunk(rows, 0), want, err_msg=f"path {path}")


def test_chunked_prefill_equals_sequential_and_pad_rows(tmp_path):
    d = GOLDEN / "fx_v1"
    toks = [(3 + i) % 16 for i in range(21)]
    with CudaModel(d) as a, CudaModel(d) as b:
        pa = a.prefill(toks)
        pb = [b.decode(t, i) for i, t in enumerate(toks)]
        for x, y in zip(pa, pb):
            np.testing.assert_array_equal(x, y)
        a.reset()
        short = a.prefill(toks[:12])
        for x, y in zip(pa[:12], short):
            np.testing.assert_array_equal(x, y)


def test_device_decode_loop_matches_records():
    rec, prompt, n = _rec("c1_v2")
    B = 3
    with CudaModel(GOLDEN / "c1_v2", batch=B) as m:
        recs = m.generate_batch([prompt] * B, 1)
        # continue with the device-resident loop from the first generated token
        m.set_tokens([recs[0]["generated"][0]] * B)
        steps = n - 1
        m.decode_async(len(prompt), steps)
        m.sync()
        h = m.history(steps)
        for b in range(B):
            assert h[:, b].tolist() == rec["argmax_per_step"][1 : 1 + steps]


def test_errors_mirror_reference():
    with CudaModel(GOLDEN / "fx_v1") as m:
        with pytest.raises(ValueError, match="max_seq"):
            m.generate(list(range(10)), 64)
        with pytest.raises(ValueError, match="empty prompt"):
            m.generate([], 3)
        with pytest.raises(ValueError, match="vocabulary"):
            m.generate([0, 99], 3)
        with pytest.raises(ValueError, match="max_seq"):
            m.run_chunk(np.zeros((16, m.dim)), 60)
        # the session stays usable after an error
        rec, prompt, n = _rec("fx_v1")
        assert m.generate(prompt, n) == rec


def test_invalid_qgraphs_are_rejected(tmp_path):
    import shutil
    src = GOLDEN / "fx_v1"
    for mutate, match in [
        (lambda g: g["ops"][0].__setitem__("sh_post", 64), "shift"),
        (lambda g: g["ops"][1].__setitem__("S", -1), "shift"),
        (lambda g: g["model"].__setitem__("prefill_m", 3), "prefill_m"),
        (lambda g: g["ops"].insert(0, {"op": "conv", "out": "x"}), "unknown qgraph op"),
        (lambda g: g["ops"][2].__setitem__("N", 31), "N"),
    ]:
        d = tmp_path / f"bad{len(list(tmp_path.iterdir()))}"
        shutil.copytree(src, d)
        g = json.loads((d / "qgraph.json").read_text())
        mutate(g)
        (d / "qgraph.json").write_text(json.dumps(g))
        with pytest.raises(ValueError, match=match):
            CudaModel(d)


def test_lanes_equal_one_session():
    """Lanes (sessions sharing one loaded model, one stream each) decode exactly like one
    session holding every sequence."""
    from llaccel_b200.cuda_backend import CudaLanes
    d = GOLDEN / "c1_v2"
    B, L, n = 8, 20, 12
    prompts = np.random.default_rng(11).integers(0, 512, (B, L)).tolist()
    with CudaModel(d, batch=B) as one:
        want = one.generate_batch(prompts, n)
    lanes = CudaLanes(d, batch=B, lanes=4)
    try:
        got = lanes.generate_batch(prompts, n)
        assert got == want
        lanes.set_tokens([r["generated"][0] for r in want])
        lanes.decode_async(L, n - 1)
        lanes.sync()
        h = lanes.history(n - 1)
        for b in range(B):
            assert h[:, b].tolist() == want[b]["argmax_per_step"][2 : 2 + n - 1]
    finally:
        lanes.close()


@pytest.mark.parametrize("name,B", [("c1_v2", 4), ("c1_v2", 20), ("qwen2_tiny", 16)])
def test_host_driven_batch_decode_matches_device_loop(name, B):
    """llx_run with batch > 1 and M = 1 (the C-ABI host loop) == the device-resident loop."""
    import ctypes as C
    from llaccel_b200.cuda_backend import _check, _p32
    o = O.OracleModel(GOLDEN / name)
    L, n = 20, 10
    prompts = np.random.default_rng(B).integers(0, o.vocab, (B, L)).tolist()
    with CudaModel(GOLDEN / name, batch=B) as m:
        recs = m.generate_batch(prompts, n)
        first = np.array([r["generated"][0] for r in recs], np.int32)
        cur = first.reshape(B, 1).copy()
        am = np.zeros(B, np.int32)
        host = []
        for i in range(n - 1):
            _check(m.lib, m.lib.llx_run(m._sess, _p32(cur), 1, L + i, None, 0, None, _p32(am)))
            host.append(am.copy())
            cur[:, 0] = am
        for b in range(B):
            assert [h[b] for h in host] == recs[b]["argmax_per_step"][2 : 2 + n - 1], b


@pytest.mark.parametrize("K,N,epi", [(8192, 8192, "resadd"), (1024, 12288, "silu"), (8192, 8192, "mul")])
def test_persistent_gemm_epilogues_match_oracle(tmp_path, K, N, epi):
    """Enough output tiles (two per SM) for the persistent double-buffered GEMM, with every
    epilogue: each CTA drains one TMEM buffer while the next tile accumulates into the other."""
    R = 1200
    d = qgraph_synth.build_linear(tmp_path / "lin", K=K, N=N, epi=epi, seed=K + N, max_seq=R)
    o = O.OracleModel(d)
    rng = np.random.default_rng(N)
    rows = rng.integers(-32768, 32768, (R, K))
    want = o.run_chunk(rows, 0)
    with CudaModel(d, max_rows=R) as m:
        np.testing.assert_array_equal(m.run_chunk(rows, 0), want)


def test_persistent_gated_prefill_matches_oracle(tmp_path):
    """A wide FFN prefilled over 20 sequences x 64 rows: the fused gate/up GEMM (silu * up +
    quant epilogue) runs on the persistent kernel; records equal the oracle's."""
    d = qgraph_synth.build(tmp_path / "g", dim=256, n_layers=1, H=4, Hkv=2, D=64, ffn=2048, vocab=300, max_seq=96,
                           seed=5)
    o = O.OracleModel(d)
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, 300, (20, 64)).tolist()
    want = [o.generate(p, 4) for p in prompts]
    with CudaModel(d, batch=20, max_rows=64) as m:
        assert m.generate_batch(prompts, 4, prefill_rows=64) == want


@pytest.mark.parametrize("D,H,Hkv,S", [(128, 8, 2, (37, 38)), (128, 8, 2, (42, 43)), (64, 14, 2, (34, 38)),
                                         (128, 4, 2, (40, 42))])
def test_long_context_batch_decode_matches_oracle(tmp_path, D, H, Hkv, S):
    """Decode attention over long slices: 96 sequences give more (sequence, KV head) pairs
    than one wave of 4-CTA clusters holds, so each pair splits its 1200+ keys over 2 CTAs of
    about 600, and the newest row (RoPE folded into the attention) lands in the last tile of
    the ring.  4 and 7 query heads per KV head take the tensor-core passes, 2 the CUDA-core
    passes with the value pass in key phases.  Ss spans a peaked and a flat softmax.
    Records equal the oracle's for every sequence, and a second run repeats them exactly."""
    L, n, B = 1200, 10, 96
    d = qgraph_synth.build(tmp_path / "g", dim=128, n_layers=1, H=H, Hkv=Hkv, D=D, ffn=64, vocab=40,
                           max_seq=L + 16, seed=21, att_S=S)
    o = O.OracleModel(d)
    rng = np.random.default_rng(21)
    distinct = rng.integers(0, o.vocab, (4, L)).tolist()
    want = [o.generate(p, n) for p in distinct]
    prompts = [distinct[b % 4] for b in range(B)]
    with CudaModel(d, batch=B, max_rows=256) as m:
        first = m.generate_batch(prompts, n, prefill_rows=256)
        for b in range(B):
            assert first[b] == want[b % 4], b
        assert m.generate_batch(prompts, n, prefill_rows=256) == first


def test_kernels_are_sm100_binaries():
    """What the CUDA runtime loaded from the library is sm_100 machine code (no JIT of PTX)."""
    import ctypes as C
    from llaccel_b200.cuda_backend import _check, load_library
    lib = load_library()
    v = C.c_int(0)
    _check(lib, lib.llx_binary_version(0, C.byref(v)))
    assert v.value == 100
