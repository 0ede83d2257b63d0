"""CPU sanity of the stress-graph builder used by the GPU parity tests."""
import numpy as np

from oracle import golden_oracle as O
import qgraph_synth


def test_stress_graphs_execute_on_the_oracle(tmp_path):
    for i, cfg in enumerate([dict(seed=1), dict(seed=3, extreme=True, fuse=False, prob_bits=8),
                             dict(seed=5, D=128, H=2, Hkv=1, dim=128, ffn=64, qk_norm=True)]):
        d = qgraph_synth.build(tmp_path / f"g{i}", **cfg)
        o = O.OracleModel(d)
        rec = o.generate(list(range(7)), 5)
        assert len(rec["generated"]) == 5
        assert np.abs(np.array(rec["logits_last_rows"])).max() > 0
