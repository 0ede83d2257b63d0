"""GPU check of llx_linear_argmax_noalloc, the entry point for callers that cannot allocate
device memory (code inside another framework's memory pool, plugin hosts with pre-sized
buffers, processes that must not grow their device footprint).  It must produce exactly the
logits and argmax of the session API on the same linear, and of the CPU oracle, on two calls
in a row (its scratch array keeps the previous call's contents, so the second call checks
the clearing), and the second call must leave the device's free memory unchanged.

The file name sorts last, so a run that stops at the first failure has run every other test
before this one."""
from __future__ import annotations

import ctypes as C
import json

import numpy as np
import pytest

from oracle import golden_oracle as O
import qgraph_synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)


def _tensor(blob, g, name, dtype, shape):
    spec = g["tensors"][name]
    n = int(np.prod(shape))
    return np.frombuffer(blob, dtype=dtype, count=n, offset=spec["offset"]).reshape(shape).copy()


@pytest.mark.parametrize("K,N,R", [(896, 1000, 300), (256, 8192, 64)])
def test_noalloc_matches_session_api(tmp_path, K, N, R):
    from llaccel_b200 import build
    build.build()
    from llaccel_b200.cuda_backend import CudaModel, _check, _p16, _p32

    d = qgraph_synth.build_linear(tmp_path / "lin", K=K, N=N, seed=K + N)
    g = json.loads((d / "qgraph.json").read_text())
    blob = np.fromfile(d / "qweights.bin", dtype=np.uint8)
    W = _tensor(blob, g, "w1", "<i1", (N, K))
    rq = _tensor(blob, g, "w1.rq", "<i4", (N, 2))
    bias = _tensor(blob, g, "w1.b", "<i4", (N,))
    rng = np.random.default_rng(R)
    rows = rng.integers(-32768, 32768, (R, K))
    q = g["ops"][0]
    A = O.vquant(rows, q["M"], q["S"]).astype(np.int8)
    vocab = g["model"]["vocab"]
    # the CPU oracle of the same graph (golden.py run_chunk + argmax over the vocabulary)
    oracle_logits = O.OracleModel(d).run_chunk(rows, 0)
    oracle_am = np.argmax(oracle_logits[:, :vocab], axis=1).astype(np.int32)

    # the existing entry point: the session API on the same graph (logits and argmax)
    with CudaModel(d, max_rows=R) as m:
        want = np.empty((R, N), np.int16)
        want_am = np.empty(R, np.int32)
        r16 = np.ascontiguousarray(rows, dtype=np.int16)
        _check(m.lib, m.lib.llx_run_rows(m._sess, _p16(r16), R, 0, _p16(want), _p32(want_am)))
        lib = m.lib

        dev = torch.device("cuda", 0)
        tA = torch.from_numpy(A).to(dev)
        tW = torch.from_numpy(W).to(dev)
        tb = torch.from_numpy(bias).to(dev)
        trq = torch.from_numpy(rq).to(dev)
        np.testing.assert_array_equal(want, oracle_logits)
        np.testing.assert_array_equal(want_am, oracle_am)
        for call in range(2):
            logits = torch.full((R, N), -7, dtype=torch.int16, device=dev)
            am = torch.full((R,), -1, dtype=torch.int32, device=dev)
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info(dev)[0]
            rc = lib.llx_linear_argmax_noalloc(tA.data_ptr(), tW.data_ptr(), tb.data_ptr(), trq.data_ptr(), R, N, K,
                                               vocab, logits.data_ptr(), am.data_ptr(), None)
            assert rc == 0, lib.llx_last_error().decode()
            if call == 1:
                # the first call may load kernel code (lazy module loading); the second must
                # not change the device's free memory at all
                assert torch.cuda.mem_get_info(dev)[0] == free0
            got, got_am = logits.cpu().numpy(), am.cpu().numpy()
            np.testing.assert_array_equal(got, want, err_msg=f"call {call}")
            np.testing.assert_array_equal(got_am, want_am, err_msg=f"call {call}")
            np.testing.assert_array_equal(got, oracle_logits, err_msg=f"call {call} vs oracle")
            np.testing.assert_array_equal(got_am, oracle_am, err_msg=f"call {call} vs oracle")
            # argmax over every channel, against the logits themselves
            rc = lib.llx_linear_argmax_noalloc(tA.data_ptr(), tW.data_ptr(), tb.data_ptr(), trq.data_ptr(), R, N, K,
                                               N, logits.data_ptr(), am.data_ptr(), None)
            assert rc == 0, lib.llx_last_error().decode()
            np.testing.assert_array_equal(am.cpu().numpy(), np.argmax(want, axis=1).astype(np.int32))


def test_noalloc_rejects_rows_beyond_its_scratch():
    from llaccel_b200.cuda_backend import load_library
    lib = load_library()
    dev = torch.device("cuda", 0)
    buf = torch.zeros(16 * 4097, dtype=torch.int8, device=dev)
    out = torch.zeros(8 * 4097, dtype=torch.int16, device=dev)
    am = torch.zeros(4097, dtype=torch.int32, device=dev)
    rc = lib.llx_linear_argmax_noalloc(buf.data_ptr(), buf.data_ptr(), None, buf.data_ptr(), 4097, 8, 16, 8,
                                       out.data_ptr(), am.data_ptr(), None)
    assert rc == 5  # LLX_ERR_RANGE
    assert "4096" in lib.llx_last_error().decode()


def test_noalloc_rejects_k_whose_sums_could_wrap():
    from llaccel_b200.cuda_backend import load_library
    lib = load_library()
    dev = torch.device("cuda", 0)
    K = 131072
    buf = torch.zeros(K * 8, dtype=torch.int8, device=dev)
    out = torch.zeros(8, dtype=torch.int16, device=dev)
    am = torch.zeros(1, dtype=torch.int32, device=dev)
    rq = torch.zeros(16, dtype=torch.int32, device=dev)
    rc = lib.llx_linear_argmax_noalloc(buf.data_ptr(), buf.data_ptr(), None, rq.data_ptr(), 1, 8, K, 8,
                                       out.data_ptr(), am.data_ptr(), None)
    assert rc == 5  # LLX_ERR_RANGE
    assert "131056" in lib.llx_last_error().decode()
