"""Tree decode steps as page-list plans on the tensor-core kernels
(BE_TREE_PAGES=1) select the same beams as the slot-list tree plans of the
general kernel, eager and from the step graph."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graph", [False, True])
def test_tree_page_plans_select_like_slot_plans(monkeypatch, graph):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    cfg = dict(TINY, head_dim=128, num_attention_heads=16, num_key_value_heads=4, hidden_size=512)
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=torch.device("cuda:0"), seed=3)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (300, 70, 17)]
    outs = []
    for pages in ("0", "1"):
        monkeypatch.setenv("BE_TREE_PAGES", pages)
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  kernel_type="fasttree", max_num_pages=1024, use_graph=graph)
        assert gen.tree_pages == (pages == "1")
        outs.append(gen.generate_ids(prompts, 8, max_new_tokens=20, num_return_sequences=8))
        if pages == "1" and graph:
            assert gen.step_graph_tpages is not None
    for a, b in zip(*outs):
        np.testing.assert_allclose([x for _, x in a], [x for _, x in b], atol=5e-2, rtol=0)
