"""Regenerate the golden fixtures under tests/golden/ from the llaccel reference.

    python tests/golden/make_fixtures.py [--reference PATH]

Needs the reference checkout (its `python/` package and its tests) and torch; it runs
only where the reference is present, never on the GPU box.  Everything it writes is
committed so that the tests need no reference at run time.

What it writes (every value below is computed by the REFERENCE's own code):
  luts.json                 SIG / EXPI / EXPF from llaccel.luts
  primitives.npz            random inputs and outputs of golden.py's primitives
  fx_v1/, fx_v2/            the reference's hand-built 1-layer qgraph fixture
                            (tests/python/test_golden_e2e.py build_fixture), unfused/fused
  c1_v1/, c1_v2/            config C1 (tiny dense Llama, seed 0) through the reference
                            importer -> calibration -> refquant, unfused/fused
  qwen2_tiny/, qwen3_tiny/  small QKV-bias (GQA rep 4) and Q/K-norm variants, fused
  for each qgraph dir: golden.json (GoldenModel.generate) and acts.npz (every named
  activation of selected launches, int32 like golden.py's --dump-acts)
The D=128 case (refquant rejects head_dim 128) is produced by llaccel_b200.artefacts
and checked by running the reference GoldenModel on it here: d128_tiny/.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def load_reference(ref: Path):
    sys.path.insert(0, str(ref / "python"))
    import llaccel.golden as G  # noqa: F401
    return G


def patch_export():
    """torch 2.11 rejects export.py's bounded Dim("T", max=max_seq) guard; an unbounded
    dynamic row dimension exports the identical graph."""
    import torch
    import llaccel.export as E

    def export_program(model, max_seq):
        model = model.eval().cpu()
        tokens = torch.zeros(1, 8, dtype=torch.long)
        with torch.no_grad():
            return torch.export.export(model, (tokens,), dynamic_shapes=({1: torch.export.Dim.DYNAMIC},))

    E.export_program = export_program
    return E


def save_golden(G, qdir: Path, prompt, n_tokens, act_launches):
    g = G.GoldenModel(qdir)
    acts: list = []
    rec = g.generate(prompt, n_tokens, acts)
    (qdir / "golden.json").write_text(json.dumps(rec))
    arrays = {}
    for i in act_launches:
        if i >= len(acts):
            continue
        step = acts[i]
        for name, arr in step["acts"].items():
            arrays[f"{i}|{step['kind']}|{step['pos']}|{name}"] = np.asarray(arr).astype(np.int32)
    np.savez_compressed(qdir / "acts.npz", **arrays)
    return rec


def export_and_quantize(G, cfg_kwargs, seed, out_base: Path, name: str, fusions, calib_n=4, calib_len=64,
                        tie=False, bias_std=0.0):
    import torch
    E = patch_export()
    from llaccel.calibrate import calibrate_tokens
    from llaccel.model import ModelConfig, TinyLlama
    from llaccel.refquant import RefQuantizer, Blob  # noqa: F401

    cfg = ModelConfig(**cfg_kwargs)
    torch.manual_seed(seed)
    model = TinyLlama(cfg).eval()
    with torch.no_grad():
        if bias_std:
            for layer in model.layers:
                for lin in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                    if lin.bias is not None:
                        lin.bias.normal_(0.0, bias_std)
        if tie:
            model.lm_head.weight.copy_(model.embed_tokens.weight)
    m = E.import_model(model, cfg)
    rng = np.random.default_rng(seed)
    seqs = [rng.integers(0, cfg.vocab, min(calib_len, cfg.max_seq)).tolist() for _ in range(calib_n)]
    calib = calibrate_tokens(m, seqs)
    weights = {n: t.detach().numpy().astype(np.float64) for n, t in m.weights}
    outs = {}
    for fusion in fusions:
        q = RefQuantizer(m.cfg, weights, calib, fusion)
        graph = q.run()
        d = out_base / (f"{name}_v2" if fusion and len(fusions) > 1 else f"{name}_v1" if len(fusions) > 1 else name)
        if d.exists():
            shutil.rmtree(d)
        d.mkdir(parents=True)
        (d / "qweights.bin").write_bytes(q.blob.bytes())
        (d / "qgraph.json").write_text(json.dumps(graph, indent=1))
        outs[fusion] = d
    # float export inputs for the artefact-generator pin (weights + calib of this model)
    return outs, m, weights, calib


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LLACCEL_REFERENCE", str(Path(__file__).resolve().parents[3] / "reference")))
    args = ap.parse_args(argv)
    ref = Path(args.reference)
    G = load_reference(ref)
    from llaccel import luts

    # ---- LUTs -------------------------------------------------------------------------------
    (HERE / "luts.json").write_text(json.dumps({
        "SIG": luts.sigmoid_lut().astype(int).tolist(),
        "EXPI": luts.exp_int_lut().astype(int).tolist(),
        "EXPF": luts.exp_frac_lut().astype(int).tolist()}))

    # ---- primitive vectors ----------------------------------------------------------------------
    rng = np.random.default_rng(20261201)
    prim = {}
    v = rng.integers(-(1 << 62), 1 << 62, 4096, dtype=np.int64)
    s = rng.integers(0, 64, 4096, dtype=np.int64)
    prim["rshr_v"], prim["rshr_s"], prim["rshr_out"] = v, s, G.rshr(v, s)
    acc = rng.integers(-(1 << 31), 1 << 31, 4096, dtype=np.int64)
    M = rng.integers(1 << 30, 1 << 31, 4096, dtype=np.int64)
    S = rng.integers(0, 64, 4096, dtype=np.int64)
    prim["rq_acc"], prim["rq_M"], prim["rq_S"] = acc, M, S
    prim["rq16_out"], prim["rq8_out"] = G.requant16(acc, M, S), G.requant8(acc, M, S)
    xs = np.arange(-32768, 32768, dtype=np.int64)
    silu_params = [(1 << 30, 30, 16), (1 << 30, 32, 17), (1 << 30, 27, 14), (1518500250, 31, 15)]
    prim["silu_params"] = np.array(silu_params, dtype=np.int64)
    prim["silu_out"] = np.stack([G.silu16(xs, *p) for p in silu_params])
    a = rng.integers(-32768, 32768, 4096, dtype=np.int64)
    b = rng.integers(-32768, 32768, 4096, dtype=np.int64)
    sh = rng.integers(0, 32, 4096, dtype=np.int64)
    prim["ew_a"], prim["ew_b"], prim["ew_sh"] = a, b, sh
    prim["vmul_out"] = np.array([G.vmul(x, y, int(k)) for x, y, k in zip(a, b, sh)], dtype=np.int64)
    prim["vadd_out"] = np.array([G.vadd(x, y, int(k)) for x, y, k in zip(a, b, sh)], dtype=np.int64)
    prim["vquant_out"] = np.array([G.vquant(x, int(m_), int(k)) for x, m_, k in zip(a, M, S)], dtype=np.int64)
    isq = np.concatenate([rng.integers(0, 1 << 48, 2048, dtype=np.int64),
                          np.array([0, 1, 2, 3, 4, (1 << 48) - 1, 1 << 47, (1 << 46) - 1, 65535**2, 65536**2], dtype=np.int64)])
    prim["isqrt_in"], prim["isqrt_out"] = isq, np.array([G.isqrt48(int(t)) for t in isq], dtype=np.int64)
    # rmsnorm rows of several widths and scales (heads share gamma)
    for K in (32, 128, 576):
        x = np.clip(rng.normal(0, rng.uniform(200, 9000), (24, K)), -32768, 32767).astype(np.int64)
        x[0] = 0
        x[1] = 1
        g = rng.integers(8000, 24000, K, dtype=np.int64)
        C = int(round(2.0**24 * np.sqrt(K)))
        prim[f"rms{K}_x"], prim[f"rms{K}_g"] = x, g
        prim[f"rms{K}_params"] = np.array([3 + K, C, 24], dtype=np.int64)
        prim[f"rms{K}_out"] = G.rmsnorm(x, g, 3 + K, C, 24)
    # rope
    for H, D in ((4, 32), (2, 64), (2, 128)):
        base = 10000.0
        inv_freq = base ** (-np.arange(0, D, 2) / D)
        ang = np.outer(np.arange(96), inv_freq)
        cos_t = np.round(np.cos(ang) * 16384).astype(np.int64)
        sin_t = np.round(np.sin(ang) * 16384).astype(np.int64)
        x = rng.integers(-32768, 32768, (5, H * D), dtype=np.int64)
        prim[f"rope{H}x{D}_x"], prim[f"rope{H}x{D}_cos"], prim[f"rope{H}x{D}_sin"] = x, cos_t, sin_t
        prim[f"rope{H}x{D}_out"] = G.rope(x, H, D, cos_t, sin_t, 37)
    # attention heads
    att_cases = []
    for i, (D, T, pb) in enumerate([(16, 1, 15), (32, 7, 15), (64, 129, 15), (64, 300, 8), (128, 257, 15),
                                    (128, 1000, 15), (16, 171, 8), (64, 4224, 15)]):
        q = rng.integers(-128, 128, D, dtype=np.int64)
        k = rng.integers(-128, 128, (T, D), dtype=np.int64)
        vv = rng.integers(-128, 128, (T, D), dtype=np.int64)
        Ms, Ss = int(rng.integers(1 << 30, 1 << 31)), int(rng.integers(20, 34))
        Mo, So = int(rng.integers(1 << 30, 1 << 31)), int(rng.integers(36, 42))
        prim[f"att{i}_q"], prim[f"att{i}_k"], prim[f"att{i}_v"] = q, k, vv
        prim[f"att{i}_params"] = np.array([Ms, Ss, Mo, So, pb], dtype=np.int64)
        prim[f"att{i}_out"] = G.attention_head(q, k, vv, Ms, Ss, Mo, So, pb)
        att_cases.append(i)
    prim["att_cases"] = np.array(att_cases)
    np.savez_compressed(HERE / "primitives.npz", **prim)

    # ---- the reference's hand-built 1-layer fixture --------------------------------------------
    spec = importlib.util.spec_from_file_location("ref_e2e", ref / "tests" / "python" / "test_golden_e2e.py")
    e2e = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(e2e)
    for name, fuse in (("fx_v1", False), ("fx_v2", True)):
        d = HERE / name
        if d.exists():
            shutil.rmtree(d)
        e2e.build_fixture(d, fuse=fuse)
        (d / "tokenizer.json").unlink(missing_ok=True)
        prompt = np.random.default_rng(0).integers(0, e2e.VOCAB, 20).tolist()
        save_golden(G, d, prompt, 12, act_launches=[0, 1, 2, 13])

    # ---- C1 through the reference pipeline -----------------------------------------------------
    c1 = dict(dim=128, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=352, vocab=512, max_seq=80,
              rope_base=10000.0, rms_eps=1e-5)
    outs, _, w, calib = export_and_quantize(G, c1, 0, HERE, "c1", (False, True))
    # keep the float export of C1 (weights as f32 + calib) to pin llaccel_b200.artefacts' quantizer
    np.savez_compressed(HERE / "c1_float.npz", **{k: v.astype(np.float32) for k, v in w.items()})
    (HERE / "c1_calib.json").write_text(json.dumps(calib, indent=1))
    prompt = np.random.default_rng(0).integers(0, 512, 16).tolist()
    for d in outs.values():
        save_golden(G, d, prompt, 64, act_launches=[0, 1, 40, 63])

    # ---- architecture variants (fused qgraphs) -------------------------------------------------
    q2 = dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=1, head_dim=64, ffn=128, vocab=80, max_seq=48,
              rope_base=1e6, rms_eps=1e-5, qkv_bias=True)
    outs, *_ = export_and_quantize(G, q2, 1, HERE, "qwen2_tiny", (True,), tie=True, bias_std=0.02)
    prompt = np.random.default_rng(1).integers(0, 80, 21).tolist()
    save_golden(G, outs[True], prompt, 20, act_launches=[0, 2, 10])
    q3 = dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn=96, vocab=96, max_seq=48,
              rope_base=1e6, rms_eps=1e-6, qk_norm=True)
    outs, *_ = export_and_quantize(G, q3, 2, HERE, "qwen3_tiny", (True,))
    prompt = np.random.default_rng(2).integers(0, 96, 17).tolist()
    save_golden(G, outs[True], prompt, 24, act_launches=[0, 1, 3, 20])

    # ---- head_dim 128: our artefact generator's qgraph, executed by the reference golden ----------
    sys.path.insert(0, str(REPO))
    from llaccel_b200 import artefacts
    d = HERE / "d128_tiny"
    if d.exists():
        shutil.rmtree(d)
    cfg = artefacts.ArchConfig(name="d128_tiny", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=256,
                               vocab=128, max_seq=64, rope_base=5e5, rms_eps=1e-5, qk_norm=True)
    artefacts.build_qgraph(cfg, d, seed=3, fusion=True, calib_seqs=2, calib_len=32, device="cpu")
    prompt = np.random.default_rng(3).integers(0, 128, 18).tolist()
    save_golden(G, d, prompt, 20, act_launches=[0, 1, 5])
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
