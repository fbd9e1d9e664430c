"""Diverse beam search through the whole B200 engine (cfg1, fp32) against the
reference engine's selections (golden e2e_cfg1_diverse.json)."""
import numpy as np
import pytest

from conftest import load_json
from test_gpu_engine import cfg1_model

pytestmark = pytest.mark.gpu


def test_cfg1_e2e_diverse_matches_reference():
    """Diverse beam search (2 groups, hamming) through the whole engine selects
    the reference engine's beams (golden e2e_cfg1_diverse.json), and several
    prompts decoded together select as each prompt alone."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import DiverseBeamSearchStrategy
    model, _, _ = cfg1_model()
    g = load_json("e2e_cfg1_diverse.json")
    gen = BeamSearchGenerator(model, None, DiverseBeamSearchStrategy(**g["strategy"]),
                              page_size=g["page_size"], max_num_pages=256)
    out = gen.generate_ids([g["prompt"]], g["beam_size"], max_length=g["max_length"],
                           num_return_sequences=g["beam_size"])[0]
    assert [s for s, _ in out] == [s for s, _ in g["final"]]
    np.testing.assert_allclose([x for _, x in out], [x for _, x in g["final"]], rtol=2e-5)
    p2 = list(reversed(g["prompt"]))
    outs = []
    for prompts in ([g["prompt"], p2], [g["prompt"]], [p2]):
        gen = BeamSearchGenerator(model, None, DiverseBeamSearchStrategy(**g["strategy"]),
                                  page_size=16, max_num_pages=512)
        outs.append(gen.generate_ids(prompts, 4, max_new_tokens=12, num_return_sequences=4))
    assert [s for s, _ in outs[0][0]] == [s for s, _ in outs[1][0]]
    assert [s for s, _ in outs[0][1]] == [s for s, _ in outs[2][0]]
