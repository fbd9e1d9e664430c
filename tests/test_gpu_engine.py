"""End-to-end parity of the B200 engine: the cfg1 tiny model in fp32 must select
the same beam tokens as the reference engine (golden e2e_cfg1.json), and the
model's logits must match the numpy oracle."""
import numpy as np
import pytest
import torch

from conftest import load_json

pytestmark = pytest.mark.gpu


def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def cfg1_model(dtype=torch.float32):
    from beam_engine_b200.llama import BeamLlama
    from beam_engine_b200.weights import random_llama_weights
    g = load_json("e2e_cfg1.json")
    cfg = g["config"]
    w = random_llama_weights(cfg, seed=0, dtype=torch.float32, device="cpu")
    return BeamLlama(cfg, w, dtype=dtype, device=dev()), g, w


def test_cfg1_prefill_logits_match_oracle():
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_state import BeamState
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from oracle.llama import OracleLlama
    from oracle.paging import OraclePageTable
    model, g, w = cfg1_model()
    gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                              max_num_pages=64)
    st = BeamState(4, gen.page_table)
    logits = gen.prefill(st, [g["prompt"]]).cpu().numpy()
    om = OracleLlama(g["config"], {k: v.numpy() for k, v in w.items()})
    table = OraclePageTable(2, 16, 64, 2, 64)
    pages = [table.allocate_block() for _ in range(4)]
    ref = om.forward(g["prompt"], list(range(64)), table, "prefill", prefill=(pages, 16))[-1]
    np.testing.assert_allclose(logits[0], ref, atol=2e-5, rtol=0)
    # and the prompt K/V landed in the same pages
    np.testing.assert_allclose(gen.page_table.kv_cache[0, :4].cpu().numpy(), table.kv[0][:4],
                               atol=2e-5, rtol=0)


@pytest.mark.parametrize("kernel_type", ["cascade"])
def test_cfg1_e2e_fp32_tokens_match_reference(kernel_type):
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    model, g, _ = cfg1_model()
    gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(length_penalty=1.0),
                              page_size=g["page_size"], kernel_type=kernel_type, max_num_pages=256)
    out = gen.generate_ids([g["prompt"]], g["beam_size"], max_length=g["max_length"],
                           num_return_sequences=g["beam_size"])[0]
    assert [s for s, _ in out] == [s for s, _ in g["final"]]
    np.testing.assert_allclose([x for _, x in out], [x for _, x in g["final"]], rtol=2e-5)


def test_cfg1_bf16_runs_and_stays_close():
    """bf16 engine on the same model: valid beams, scores near the fp32 run."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    model, g, _ = cfg1_model(torch.bfloat16)
    gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                              max_num_pages=256)
    out = gen.generate_ids([g["prompt"]], 4, max_length=96, num_return_sequences=4)[0]
    assert len(out) == 4 and all(len(s) == 96 for s, _ in out)
    assert all(s[:64] == g["prompt"] for s, _ in out)
    ref = np.asarray([x for _, x in g["final"]])
    assert np.abs(np.asarray([x for _, x in out]) - ref).max() < 0.05


def test_multi_prompt_batch_matches_single_runs():
    """Two prompts decoded together give the same beams as each prompt alone."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    model, g, _ = cfg1_model()
    p1 = g["prompt"]
    p2 = list(reversed(g["prompt"]))
    outs = []
    for prompts in ([p1, p2], [p1], [p2]):
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  max_num_pages=512)
        outs.append(gen.generate_ids(prompts, 4, max_new_tokens=20, num_return_sequences=4))
    assert [s for s, _ in outs[0][0]] == [s for s, _ in outs[1][0]]
    assert [s for s, _ in outs[0][1]] == [s for s, _ in outs[2][0]]


@pytest.mark.parametrize("tiles", ["1", "0"])
def test_graph_step_matches_eager_bf16(monkeypatch, tiles):
    """The CUDA-graph decode step (fixed-shape attention launches, plan on the
    device) selects the same beams as the eager step, on the beam-tile kernel
    (default) and on the work-item kernels (BE_ATTN_TILES=0)."""
    monkeypatch.setenv("BE_ATTN_TILES", tiles)
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    cfg = dict(TINY, head_dim=128, num_attention_heads=4, num_key_value_heads=2, hidden_size=512)
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=dev(), seed=3)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (70,), generator=g).tolist() for _ in range(3)]
    outs = []
    for graph in (False, True):
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  max_num_pages=512, use_graph=graph)
        outs.append(gen.generate_ids(prompts, 8, max_new_tokens=24, num_return_sequences=8))
        assert gen.use_graph == graph
        assert gen.use_tiles == (tiles == "1")
        if graph:
            sg = gen.step_graph_tiles if tiles == "1" else gen.step_graph
            assert sg is not None and sg.graph is not None
    for a, b in zip(*outs):
        assert [s for s, _ in a] == [s for s, _ in b]
        np.testing.assert_allclose([x for _, x in a], [x for _, x in b], rtol=1e-6)


def test_auto_picker_runs_and_agrees_when_it_picks_cascade():
    """kernel_type="auto" decides per step; its beams equal the cascade run's
    when every pick was cascade, and equal the tree run's when every pick was
    the tree (fp32, cfg1)."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    model, g, _ = cfg1_model()
    runs = {}
    for kt in ("auto", "cascade", "fasttree"):
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  kernel_type=kt, max_num_pages=512)
        runs[kt] = (gen.generate_ids([g["prompt"]], 4, max_new_tokens=16, num_return_sequences=4)[0],
                    list(gen.picks))
    out, picks = runs["auto"]
    assert len(picks) == 15 and set(picks) <= {"cascade", "fasttree"}
    if set(picks) == {"cascade"}:
        assert [s for s, _ in out] == [s for s, _ in runs["cascade"][0]]
    if set(picks) == {"fasttree"}:
        assert [s for s, _ in out] == [s for s, _ in runs["fasttree"][0]]


@pytest.mark.parametrize("pages", ["1", "0"])
def test_tree_graph_step_matches_eager_bf16(monkeypatch, pages):
    """Tree-attention decode steps replayed from a CUDA graph (page-list plans on
    the tensor-core kernels by default, slot-list plans through the fixed-grid
    kernel with BE_TREE_PAGES=0) select the same beams as eager tree steps."""
    monkeypatch.setenv("BE_TREE_PAGES", pages)
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    cfg = dict(TINY, head_dim=128, num_attention_heads=4, num_key_value_heads=2, hidden_size=512)
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=dev(), seed=3)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (70,), generator=g).tolist() for _ in range(3)]
    outs = []
    for graph in (False, True):
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  kernel_type="fasttree", max_num_pages=512, use_graph=graph)
        outs.append(gen.generate_ids(prompts, 8, max_new_tokens=12, num_return_sequences=8))
        assert gen.use_graph_tree == graph
        if graph:
            sg = gen.step_graph_tpages if pages == "1" else gen.step_graph_tree
            assert sg is not None and sg.graph is not None
    for a, b in zip(*outs):
        assert [s for s, _ in a] == [s for s, _ in b]
        np.testing.assert_allclose([x for _, x in a], [x for _, x in b], rtol=1e-6)
