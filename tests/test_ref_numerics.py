"""Cross-checks the numpy oracle against the reference's own C++ numerics contract
(include/llaccel/numerics.h compiled by oracle/Makefile into oracle/_ref/)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import REPO
from oracle import golden_oracle as O

LIB = REPO / "oracle" / "_ref" / "libnumerics_ref.so"
pytestmark = pytest.mark.skipif(not LIB.exists(), reason="reference numerics shim not built (make -C oracle)")


@pytest.fixture(scope="module")
def ref():
    lib = C.CDLL(str(LIB))
    i64, u32, u64, i32 = C.c_int64, C.c_uint32, C.c_uint64, C.c_int32
    for name, res, args in [("ref_rshr", i64, [i64, u32]), ("ref_mulshift", i64, [i64, u32, u32]),
                            ("ref_isqrt48", u32, [u64]), ("ref_requant16", i64, [i32, i32, i32]),
                            ("ref_silu16", i64, [i64, u32, u32, u32]), ("ref_vmul", i64, [i64, i64, u32]),
                            ("ref_vadd", i64, [i64, i64, u32]), ("ref_vquant", i64, [i64, u32, u32])]:
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    lib.ref_rmsnorm.restype = None
    lib.ref_rope.restype = None
    lib.ref_attention_head.restype = None
    return lib


def test_scalar_primitives(ref):
    rng = np.random.default_rng(11)
    for v, s in zip(rng.integers(-(1 << 62), 1 << 62, 500), rng.integers(0, 64, 500)):
        assert ref.ref_rshr(int(v), int(s)) == int(O.rshr(v, s))
    for x, M, S in zip(rng.integers(-(1 << 31), 1 << 31, 500), rng.integers(1 << 30, 1 << 31, 500),
                       rng.integers(0, 64, 500)):
        assert ref.ref_requant16(int(x), int(M), int(S)) == int(O.requant16(x, M, S))
        assert ref.ref_vquant(int(x) >> 16, int(M), int(S)) == int(O.vquant(int(x) >> 16, M, S))
    for t in list(rng.integers(0, 1 << 48, 300)) + [0, 1, (1 << 48) - 1]:
        assert ref.ref_isqrt48(int(t)) == O.isqrt48(int(t))
    for x in range(-32768, 32768, 37):
        assert ref.ref_silu16(x, 1 << 30, 30, 16) == int(O.silu16(x, 1 << 30, 30, 16))
        assert ref.ref_silu16(x, 1 << 30, 33, 18) == int(O.silu16(x, 1 << 30, 33, 18))
    for a, b, s in zip(rng.integers(-32768, 32768, 300), rng.integers(-32768, 32768, 300), rng.integers(0, 20, 300)):
        assert ref.ref_vmul(int(a), int(b), int(s)) == int(O.vmul(a, b, s))
        assert ref.ref_vadd(int(a), int(b), int(s)) == int(O.vadd(a, b, s))


def test_row_kernels(ref):
    rng = np.random.default_rng(12)
    for K in (16, 128, 896):
        x = np.clip(rng.normal(0, 3000, K), -32768, 32767).astype(np.int16)
        g = rng.integers(8000, 30000, K).astype(np.int16)
        y = np.zeros(K, np.int16)
        C_ = int(round(2.0**22 * np.sqrt(K)))
        ref.ref_rmsnorm(x.ctypes.data_as(C.c_void_p), g.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p),
                        C.c_uint32(K), C.c_uint32(77), C.c_uint32(C_), C.c_uint32(22))
        np.testing.assert_array_equal(y, O.rmsnorm(x[None].astype(np.int64), g, 77, C_, 22)[0])
    H, D = 3, 64
    x = rng.integers(-32768, 32768, H * D).astype(np.int16)
    cs = rng.integers(-16384, 16385, (2, D // 2)).astype(np.int16)
    y = np.zeros(H * D, np.int16)
    ref.ref_rope(x.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), C.c_uint32(H), C.c_uint32(D),
                 cs[0].ctypes.data_as(C.c_void_p), cs[1].ctypes.data_as(C.c_void_p))
    np.testing.assert_array_equal(y, O.rope(x[None].astype(np.int64), H, D, cs[:1], cs[1:], 0)[0])


@pytest.mark.parametrize("D,T,wide", [(16, 1, 1), (32, 50, 1), (64, 256, 0), (128, 700, 1), (64, 4224, 1)])
def test_attention_head(ref, D, T, wide):
    rng = np.random.default_rng(D * T)
    q = rng.integers(-128, 128, D).astype(np.int8)
    k = rng.integers(-128, 128, (T, D)).astype(np.int8)
    v = rng.integers(-128, 128, (T, D)).astype(np.int8)
    out = np.zeros(D, np.int8)
    Ms, Ss, Mo, So = 1500000000, 28, 1300000000, 39
    ref.ref_attention_head(q.ctypes.data_as(C.c_void_p), k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p),
                           C.c_uint32(D), C.c_uint32(T), C.c_uint32(Ms), C.c_uint32(Ss), C.c_uint32(Mo),
                           C.c_uint32(So), out.ctypes.data_as(C.c_void_p), C.c_int(wide))
    np.testing.assert_array_equal(out, O.attention_head(q, k, v, Ms, Ss, Mo, So, 15 if wide else 8))
