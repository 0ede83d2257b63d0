"""GPU tests of tensor parallelism (rank graphs from llaccel_b200.tp.shard).

* one GPU: a world-1 rank graph runs the row-split linears as int32 partial sums
  (tensor-core and CUDA-core GEMMs), an all-reduce that is a no-op, and the requant kernel;
  records must equal the unsharded golden bit for bit;
* two GPUs (skipped with fewer): two processes, one per GPU, NCCL all-reduces of the
  partial sums and of the argmax keys inside the captured decode graph, logits all-gathered
  on request; both ranks' records must equal the golden / oracle records.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import pickle
import time

import numpy as np
import pytest

from conftest import GOLDEN
from oracle.golden_oracle import OracleModel

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)


def _build():
    from llaccel_b200 import build
    build.build()


@pytest.mark.parametrize("name", ["c1_v2", "qwen3_tiny", "d128_tiny"])
@pytest.mark.parametrize("gemm_path", [0, 1, 3, 4])
def test_tp1_rank_graph_matches_golden(tmp_path, name, gemm_path):
    _build()
    from llaccel_b200 import tp
    from llaccel_b200.cuda_backend import CudaModel
    tp.shard(GOLDEN / name, tmp_path / "r0", 0, 1)
    rec = json.loads((GOLDEN / name / "golden.json").read_text())
    with CudaModel(tmp_path / "r0", gemm_path=gemm_path) as m:
        assert m.generate(rec["prompt_tokens"], len(rec["generated"])) == rec
        assert m.generate(rec["prompt_tokens"], len(rec["generated"]), fast=False) == rec


def test_tp1_batch_prefill_rows(tmp_path):
    _build()
    from llaccel_b200 import tp
    from llaccel_b200.cuda_backend import CudaModel
    src = GOLDEN / "c1_v2"
    tp.shard(src, tmp_path / "r0", 0, 1)
    ref = OracleModel(src)
    rng = np.random.default_rng(11)
    prompts = rng.integers(0, ref.vocab, (20, 37)).tolist()
    want = [ref.generate(p, 9) for p in prompts]
    with CudaModel(tmp_path / "r0", batch=20, max_rows=48) as m:
        for pr in (None, 0, 16):
            assert m.generate_batch(prompts, 9, prefill_rows=pr) == want


# ---- two ranks -----------------------------------------------------------------------------
def _rank_main(rank, world, dirs, uid_path, out_path, jobs):
    """One tensor-parallel rank: joins the group, runs `jobs`, pickles its results."""
    try:
        import torch as _t
        _t.cuda.set_device(rank)
        from llaccel_b200.cuda_backend import CudaModel, tp_unique_id

        def unique_id(j):
            # a communicator per job: rank 0 makes a fresh id, the others read it
            path = f"{uid_path}.{j}"
            if rank == 0:
                with open(path + ".tmp", "wb") as f:
                    f.write(tp_unique_id())
                os.replace(path + ".tmp", path)
            t0 = time.time()
            while not os.path.exists(path):
                if time.time() - t0 > 60:
                    raise TimeoutError("no NCCL unique id from rank 0")
                time.sleep(0.05)
            return open(path, "rb").read()

        results = []
        for j, (kind, kw) in enumerate(jobs):
            uid = unique_id(j)
            with CudaModel(dirs[rank], device=rank, tp=(rank, world, uid), **kw["model"]) as m:
                if kind == "generate":
                    results.append([m.generate(p, kw["n"], fast=kw.get("fast", True)) for p in kw["prompts"]])
                elif kind == "batch":
                    results.append(m.generate_batch(kw["prompts"], kw["n"], prefill_rows=kw.get("prefill_rows")))
                elif kind == "decode_loop":
                    L = len(kw["prompts"][0])
                    # prefill only: the last prefill argmax is the first generated token
                    recs = m.generate_batch(kw["prompts"], 0, with_logits=False)
                    m.set_tokens([r["argmax_per_step"][-1] for r in recs])
                    m.decode_async(L, kw["n"])
                    m.sync()
                    results.append(m.history(kw["n"]).tolist())
        with open(out_path, "wb") as f:
            pickle.dump(("ok", results), f)
    except BaseException as e:  # pragma: no cover - reported to the parent
        with open(out_path, "wb") as f:
            pickle.dump(("error", repr(e)), f)


def _run_group(tmp_path, src, world, jobs, timeout=300):
    from llaccel_b200 import tp
    dirs = []
    for r in range(world):
        tp.shard(src, tmp_path / f"r{r}", r, world)
        dirs.append(str(tmp_path / f"r{r}"))
    ctx = mp.get_context("spawn")
    uid_path = str(tmp_path / "uid.bin")
    outs = [str(tmp_path / f"out{r}.pkl") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, dirs, uid_path, outs[r], jobs)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + timeout
    for p in procs:
        p.join(max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(10)
    assert not alive, "a tensor-parallel rank did not finish in time"
    res = []
    for r, o in enumerate(outs):
        status, val = pickle.load(open(o, "rb"))
        assert status == "ok", f"rank {r}: {val}"
        res.append(val)
    return res


needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@needs2
def test_tp2_generate_matches_golden(tmp_path):
    _build()
    for name in ("c1_v2", "qwen3_tiny", "d128_tiny"):
        src = GOLDEN / name
        rec = json.loads((src / "golden.json").read_text())
        jobs = [("generate", {"model": {}, "prompts": [rec["prompt_tokens"]], "n": len(rec["generated"])}),
                ("generate", {"model": {"gemm_path": 1}, "prompts": [rec["prompt_tokens"]],
                              "n": len(rec["generated"]), "fast": False})]
        res = _run_group(tmp_path / name, src, 2, jobs)
        for r in range(2):
            for j in range(len(jobs)):
                assert res[r][j][0] == rec, f"{name} rank {r} job {j}"


@needs2
def test_tp2_batch_and_decode_loop(tmp_path):
    _build()
    src = GOLDEN / "c1_v2"
    ref = OracleModel(src)
    rng = np.random.default_rng(3)
    prompts = rng.integers(0, ref.vocab, (24, 33)).tolist()
    want = [ref.generate(p, 12) for p in prompts]
    jobs = [("batch", {"model": {"batch": 24, "max_rows": 48}, "prompts": prompts, "n": 12, "prefill_rows": 16}),
            ("batch", {"model": {"batch": 24, "max_rows": 48}, "prompts": prompts, "n": 12, "prefill_rows": 0}),
            ("decode_loop", {"model": {"batch": 24, "max_rows": 48}, "prompts": prompts, "n": 10})]
    res = _run_group(tmp_path, src, 2, jobs)
    hist_want = np.array([w["generated"][1:11] for w in want]).T.tolist()
    for r in range(2):
        assert res[r][0] == want
        assert res[r][1] == want
        assert res[r][2] == hist_want
