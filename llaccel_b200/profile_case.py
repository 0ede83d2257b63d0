"""A small decode case for profilers: one of the bench configs with a short prompt, so a
capture holds a few GB on the device at most and ends by itself.

    python -m llaccel_b200.profile_case --config c3 --batch 128 --prompt 512 --max-rows 64 --decode 3

Generates (or reuses) the config's artefact under --artefacts, prefills `batch` random
prompts of `prompt` tokens in launches of `max-rows` rows per sequence (default: the whole
prompt in one launch), then runs `decode` device-resident decode launches and prints the
first sequence's tokens.  With --max-rows 64 the bench's decode shapes (128 sequences at
context ~512) hold about 1.3 GB on the device, so a capture stays small.  Tensor-core GEMM
launches before the first decode launch: (prefill launches) x (4 per layer + 1).

--layers N keeps the config's shapes but only N layers (the artefact is generated under its
own name): every kernel of a layer runs with the full config's shapes while the device holds
a fraction of the model, e.g. C5 attention at 256 sequences and context 1024 with 2 layers
(about 2.5 GB instead of 30).
"""
from __future__ import annotations

import argparse
import os
import tempfile
from pathlib import Path

import numpy as np


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c3")
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--decode", type=int, default=3)
    ap.add_argument("--max-rows", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0, help="keep only this many layers (0: all)")
    ap.add_argument("--artefacts", default=os.environ.get("LLX_ARTEFACTS", str(Path(tempfile.gettempdir()) / "llx_artefacts")))
    a = ap.parse_args(argv)
    from llaccel_b200 import artefacts as A, build
    build.build()
    from llaccel_b200.cuda_backend import CudaModel
    if a.layers:
        import dataclasses
        cfg = dataclasses.replace(A.CONFIGS[a.config], name=f"{a.config}_l{a.layers}", n_layers=a.layers)
        d = Path(a.artefacts) / f"{cfg.name}_s0_v2"
        if not (d / "manifest.json").exists():
            A.build_qgraph(cfg, d, seed=0, fusion=True, device="cuda")
    else:
        d = A.ensure_artefact(a.config, a.artefacts, seed=0, fusion=True, device="cuda")
    rows = a.max_rows or a.prompt
    m = CudaModel(d, batch=a.batch, max_rows=rows)
    prompts = np.random.default_rng(0).integers(0, A.CONFIGS[a.config].vocab, (a.batch, a.prompt)).tolist()
    recs = m.generate_batch(prompts, 0, with_logits=False, prefill_rows=rows)
    m.set_tokens([r["argmax_per_step"][-1] for r in recs])
    m.decode_async(a.prompt, a.decode)
    m.sync()
    print("ok", m.history(a.decode)[:, 0].tolist())
    m.close()


if __name__ == "__main__":
    main()
