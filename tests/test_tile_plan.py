"""Beam-tile plans (be_tile_plan, be_beam_decode_tiles) on CPU: every query of a
tile plan must attend exactly the tokens -- with the same multiplicity -- that
the work-item cascade plan (be_cascade_plan, the restatement of FlashInfer's
MultiLevelCascadeAttentionWrapper semantics used at modeling_llama.py:733-755)
makes it attend, along the reference's own trajectories (forks, frees, uneven
trees whose pages the reference's cascade lists twice) and on several prompts
decoded together.  Pieces must partition each tile's entries."""
import ctypes as C

import numpy as np
import pytest

from beam_engine_b200 import _lib
from beam_engine_b200.beam_state import BeamState
from beam_engine_b200.cascade import cascade_plan_host, tile_plan_host
from test_host_native import cpu_table, plan_token_sets


def tile_arrays(plan, info):
    tiles = plan[info.off_tiles:info.off_tiles + 8 * info.n_tiles].reshape(-1, 8)
    pieces = plan[info.off_pieces:info.off_pieces + 24 * info.n_pieces].reshape(-1, 24)
    ents = plan[info.off_entries:info.off_entries + 4 * info.n_entries].reshape(-1, 4)
    return tiles, pieces, ents


def tile_token_sets(plan, info, ps):
    """Per query: the sorted slot ids (page * ps + i) the tile plan makes it
    attend, read through the pieces (so an entry outside every piece is lost
    and one in two pieces counts twice)."""
    tiles, pieces, ents = tile_arrays(plan, info)
    out = {}
    for t, b, e, *_ in pieces:
        q0 = tiles[t][0]
        for page, ntok, lo, hi in ents[b:e]:
            toks = [int(page) * ps + i for i in range(ntok)]
            for q in range(lo, hi):
                out.setdefault(int(q0 + q), []).extend(toks)
    return {q: sorted(v) for q, v in out.items()}


def check_structure(plan, info, g):
    tiles, pieces, ents = tile_arrays(plan, info)
    assert info.n_queries == sum(int(t[1]) for t in tiles)
    nxt, part = 0, 0
    for ti, t in enumerate(tiles):
        q_begin, q_len, p0, npc, pb = (int(x) for x in t[:5])
        assert q_begin == nxt and 1 <= q_len and q_len * g <= info.tile_rows
        nxt += q_len
        own = pieces[p0:p0 + npc]
        assert (own[:, 0] == ti).all() and own[:, 3].tolist() == list(range(npc))
        # each piece repeats its tile's queries, piece count and partial base
        assert (own[:, 4:8] == np.array([q_begin, q_len, npc, pb])).all()
        for pc in own:                  # the first four entries ride in the piece record
            first = pc[8:24].reshape(4, 4)
            n = min(4, int(pc[2] - pc[1]))
            assert (first[:n] == ents[pc[1]:pc[1] + n]).all() and (first[n:] == 0).all()
        # contiguous, in order, covering the tile's entries
        for a, b in zip(own[:-1], own[1:]):
            assert a[2] == b[1]
        if info.cluster > 1:          # clusters merge on chip: no partial slots
            assert npc == info.cluster and pb == -1
        elif npc > 1:
            assert pb == part
            part += npc
        else:
            assert pb == -1
        for _, b, e, *_ in own:
            for page, ntok, lo, hi in ents[b:e]:
                assert 0 < ntok <= info.page_size and 0 <= lo < hi <= q_len
            if info.cluster <= 1:
                assert e > b or npc == 1     # only cluster plans carry empty pieces
    assert info.n_part_pieces == part
    assert info.off_pieces == 32
    assert info.max_piece_entries == max(int(p[2] - p[1]) for p in pieces)
    assert info.n_pieces == len(pieces)


def check_levels(levels, nq, ps, hq, hkv, **kw):
    got = tile_plan_host(levels, nq, ps, hq, hkv, **kw)
    assert got is not None
    info, plan = got
    check_structure(plan, info, hq // hkv)
    ref_info, ref_plan = cascade_plan_host(levels, nq, ps, hq, hkv)
    want = plan_token_sets(ref_plan, ref_info, ps)
    assert tile_token_sets(plan, info, ps) == want
    _, _, ents = tile_arrays(plan, info)
    assert info.total_tokens == int(ents[:, 1].sum()) if len(ents) else info.total_tokens == 0
    return info


@pytest.mark.parametrize("case", ["ps4_w4", "ps16_w8", "ps8_w6_churn", "ps16_w16"])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (64, 2)])
def test_tile_plans_attend_what_cascade_plans_attend(trajectories, case, hq, hkv):
    rec = trajectories[case]
    cs = rec["case"]
    ps = cs["ps"]
    for step in rec["steps"]:
        levels = step["cascade"]["levels"]
        nq = len(step["cascade"]["query"])
        for pieces in (1, 7, 300):
            check_levels(levels, nq, ps, hq, hkv, pieces=pieces, cluster=0)
        for cl in (2, 5, 16, -1):
            check_levels(levels, nq, ps, hq, hkv, pieces=37, cluster=cl)


def test_several_prompts_and_small_tiles():
    """Three prompts of 12 beams with g = 8: 96 rows -> tiles of 8 queries at
    tile_rows 64 (a prompt's group spans two tiles), one tile per prompt at 128."""
    rng = np.random.default_rng(4)
    W = 12
    pt = cpu_table(16, 4096)
    bs = BeamState(W, pt)
    for p in range(3):
        bs.add_root_sequence(rng.integers(0, 500, 100 + 37 * p).tolist())
    bs.update_native(bs.leaves, np.arange(4, dtype=np.int32) * W,
                     rng.integers(0, 500, 3 * W).astype(np.int32), -rng.random(3 * W))
    for step in range(20):
        n = len(bs.leaves)
        levels = bs.cascade_levels()
        for rows in (64, 128):
            for cl in (0, 4):
                info = check_levels(levels, n, 16, 64, 8, tile_rows=rows, cluster=cl)
                assert info.n_tiles == (6 if rows == 64 else 3)
                assert info.cluster == cl
        cnt = np.zeros(n, np.int32)
        for p in range(3):
            c = np.zeros(W, np.int32)
            c[: W // 2] = 2
            rng.shuffle(c)
            cnt[p * W:(p + 1) * W] = c
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        bs.update_native(bs.leaves, ptr, rng.integers(0, 500, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))


def test_prefill_and_bad_shapes_are_refused():
    # a causal group of several queries is a prompt, not a decode step
    lv = [dict(qo_indptr=[0, 5], kv_indptr=[0, 1], kv_indices=[3], kv_last_page_len=[5])]
    assert tile_plan_host(lv, 5, 16, 8, 2, causal=True) is None
    assert tile_plan_host(lv, 5, 16, 8, 2, causal=False, cluster=0) is not None
    # group size above the tile height
    lv1 = [dict(qo_indptr=[0, 1], kv_indptr=[0, 1], kv_indices=[3], kv_last_page_len=[5])]
    assert tile_plan_host(lv1, 1, 16, 256, 1, tile_rows=128) is None
    info = _lib.TilePlanInfo()
    arr = (_lib.P32 * 1)()
    rc = _lib.lib().be_tile_plan(0, arr, arr, arr, arr, None, 0, 16, 8, 2, 1, 96, 4, 0, None, 0,
                                 C.byref(info))
    assert rc == _lib.BE_EINVAL
    rc = _lib.lib().be_tile_plan(0, arr, arr, arr, arr, None, 0, 16, 8, 2, 1, 64, 4, 17, None, 0,
                                 C.byref(info))
    assert rc == _lib.BE_EINVAL                  # clusters hold at most 16 CTAs


def test_empty_groups_and_queries_without_pages():
    """Queries whose groups have no pages still get a tile (and an empty piece),
    so the kernel writes their zero output; zero-length last pages add nothing."""
    lv = [dict(qo_indptr=[0, 2, 4], kv_indptr=[0, 0, 2], kv_indices=[7, 9],
               kv_last_page_len=[0, 0]),
          dict(qo_indptr=[0, 1, 2, 3, 4], kv_indptr=[0, 1, 1, 2, 3], kv_indices=[11, 12, 13],
               kv_last_page_len=[3, 0, 16, 0])]
    info = check_levels(lv, 4, 16, 8, 2, cluster=0)
    plan = tile_plan_host(lv, 4, 16, 8, 2, cluster=0)[1]
    tiles, pieces, ents = tile_arrays(plan, info)
    assert info.n_tiles == 2 and sum(int(t[3]) for t in tiles) == info.n_pieces
    # page 9 (last page of group 2 at level 0, length 0) never appears
    assert 9 not in ents[:, 0].tolist()


def test_decode_tiles_match_separate_calls():
    """be_beam_decode_tiles writes the step inputs and exactly the tile plan of
    step_inputs + cascade_levels + be_tile_plan."""
    rng = np.random.default_rng(3)
    pt = cpu_table(16, 4096)
    W = 16
    bs = BeamState(W, pt)
    bs.defer_copies = True
    for p in range(2):
        bs.add_root_sequence(rng.integers(0, 500, 200 + 13 * p).tolist())
    bs.update_native(bs.leaves, np.arange(3, dtype=np.int32) * W,
                     rng.integers(0, 500, 2 * W).astype(np.int32), -rng.random(2 * W))
    for step in range(10):
        n = len(bs.leaves)
        q, wp, wpos, pos = bs.step_inputs()
        info_ref, plan_ref = tile_plan_host(bs.cascade_levels(), n, 16, 32, 8, tile_rows=64,
                                            pieces=20, cluster=-1)
        off = -(-4 * n // 32) * 32
        buf = np.full(off + (1 << 16), -7, np.int32)
        info = _lib.TilePlanInfo()
        leaves = np.ascontiguousarray(bs.leaves, np.int32)
        rc = _lib.lib().be_beam_decode_tiles(pt._trie, n, _lib.ptr32(leaves), 32, 8, 64, 20, -1,
                                             C.c_void_p(buf.ctypes.data), len(buf), off,
                                             C.byref(info))
        assert rc == _lib.BE_OK
        assert buf[:n].tolist() == list(q) and buf[n:2 * n].tolist() == list(pos)
        assert buf[2 * n:3 * n].tolist() == list(wp) and buf[3 * n:4 * n].tolist() == list(wpos)
        assert info.total_ints == info_ref.total_ints
        # about 20 pieces over the tiles: a cluster per (tile, KV head), a power
        # of two up to 8 (16 from 32 pieces per tile)
        per = 20 // info.n_tiles
        want = 16 if per >= 32 else 1 << (min(per, 8).bit_length() - 1)
        assert info.cluster == info_ref.cluster == (want if want > 1 else 0)
        assert buf[off:off + info.total_ints].tolist() == plan_ref[:info.total_ints].tolist()
        cnt = np.zeros(n, np.int32)
        cnt[rng.choice(n, n // 2, replace=False)] = 2
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        seg_ptr = ptr  # every candidate's children
        bs.update_native(bs.leaves, seg_ptr, rng.integers(0, 500, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))


def _decode_state(prompts, prompt_len, beams, steps, seed=0):
    """Beam trie after `steps` selections in which half of every prompt's
    beams fork in two and the other half end."""
    rng = np.random.default_rng(seed)
    bs = BeamState(beams, cpu_table(16, 65536))
    for _ in range(prompts):
        bs.add_root_sequence(rng.integers(0, 1000, prompt_len).tolist())
    bs.update_native(bs.leaves, np.arange(prompts + 1, dtype=np.int32) * beams,
                     rng.integers(0, 1000, prompts * beams).astype(np.int32),
                     -rng.random(prompts * beams))
    for _ in range(steps):
        cnt = np.zeros(len(bs.leaves), np.int32)
        for p in range(prompts):
            c = np.zeros(beams, np.int32)
            c[: beams // 2] = 2
            rng.shuffle(c)
            cnt[p * beams:(p + 1) * beams] = c
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        bs.update_native(bs.leaves, ptr, rng.integers(0, 1000, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))
    return bs


@pytest.mark.parametrize("prompts,prompt_len,beams,tp,cluster", [
    (8, 1024, 16, 1, 4), (8, 1024, 16, 2, 8), (8, 1024, 16, 4, 8), (8, 1024, 16, 8, 16),
    (1, 4096, 32, 1, 0), (1, 4096, 32, 8, 0)])
def test_auto_cluster_choice(prompts, prompt_len, beams, tp, cluster):
    """The planner's own cluster size: power-of-two clusters sized to the pieces
    a tile gets, except that one long tile (a single prompt with a long prefix),
    which a 16-CTA cluster would cap at 16 pieces, takes the merge kernel's form
    and keeps all its pieces."""
    from beam_engine_b200.cascade import target_pieces
    bs = _decode_state(prompts, prompt_len, beams, 20)
    hq, hkv = 32 // tp, 8 // tp
    info, _ = tile_plan_host(bs.cascade_levels(), len(bs.leaves), 16, hq, hkv, num_sms=148,
                             pieces=target_pieces(148, hkv))
    assert info.cluster == cluster
    if cluster == 0:
        assert info.n_pieces > 16 * info.n_tiles
