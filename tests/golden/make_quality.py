"""Quality fixture for config C1: the reference's fp32 model, teacher-forced on the C1 golden
token stream, and the reference's own quality metrics for that record.

    python tests/golden/make_quality.py [--reference PATH]

Runs only where the reference is present. It writes `c1_quality.npz`:
  fp32_logits   [T][vocab] float32: llaccel.verify.fp32_logits_teacher_forced on the C1
                TinyLlama (seed 0, the model make_fixtures.py exports) over prompt + generated
                tokens of c1_v2/golden.json;
  cos, top1_golden, top1_fp32   per recorded step, computed with llaccel.verify.cosine
                exactly as compare_models does (verify.py:45-60).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(HERE.parents[2] / "reference"))
    a = ap.parse_args(argv)
    ref = Path(a.reference)
    sys.path.insert(0, str(ref / "python"))
    sys.path.insert(0, str(HERE))
    import torch
    from llaccel.model import ModelConfig, TinyLlama
    from llaccel.verify import cosine, fp32_logits_teacher_forced
    import make_fixtures as MF

    # the C1 float model exactly as make_fixtures.export_and_quantize builds it
    c1 = dict(dim=128, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=352, vocab=512, max_seq=80,
              rope_base=10000.0, rms_eps=1e-5)
    torch.manual_seed(0)
    model = TinyLlama(ModelConfig(**c1)).eval()
    # the committed float export must be this model's weights
    w = dict(np.load(HERE / "c1_float.npz"))
    E = MF.patch_export()
    m = E.import_model(model, ModelConfig(**c1))
    for n, t in m.weights:
        np.testing.assert_array_equal(t.detach().numpy().astype(np.float32), w[n])

    rec = json.loads((HERE / "c1_v2" / "golden.json").read_text())
    seq = rec["prompt_tokens"] + rec["generated"]
    fp = fp32_logits_teacher_forced(model, seq)
    vocab = rec["model"]["vocab"]
    E_LOGIT = rec["model"]["E_LOGIT"]
    cos, tg, tf = [], [], []
    for j, step in enumerate(rec["steps"]):
        ctx_len = step["pos"] + step["valid_rows"]
        gl = np.array(rec["logits_last_rows"][j][:vocab], dtype=np.float64) * 2.0 ** E_LOGIT
        fl = fp[ctx_len - 1]
        cos.append(cosine(gl, fl))
        tg.append(int(np.argmax(gl)))
        tf.append(int(np.argmax(fl)))
    np.savez_compressed(HERE / "c1_quality.npz", fp32_logits=fp.astype(np.float32), cos=np.array(cos),
                        top1_golden=np.array(tg), top1_fp32=np.array(tf))
    print("c1_quality.npz:", len(cos), "steps, top-1 agreement", np.mean(np.array(tg) == np.array(tf)),
          "mean cosine", float(np.mean(cos)))


if __name__ == "__main__":
    main()
