"""The prefill's position triple from token ids (Prompt::thw_indexes,
src/u15-prompt.cc:349-386 of the reference) through the C ABI, on the CPU:
hand-derived cases, the properties the reference's prompt test asserts
(tests/u15-prompt-test.cc:190-246: context tokens share one t, the
generated image sits at max(t) + 1, h / w restart per image), and the
restated rule on random id sequences. The reference's own fixtures for this
test need its tokenizer and golden files, which are absent, so the rule is
pinned by these cases rather than by reference output."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

IMG, CTX, END = 151665, 151667, 151666   # <img>, <IMG_CONTEXT>, </img>


def thw(ids, grids):
    import u15b200
    from u15b200._lib import check
    ids = np.ascontiguousarray(ids, np.int32)
    g = np.ascontiguousarray(np.array(grids, np.int32).reshape(-1))
    t, h, w = (np.zeros(len(ids), np.int32) for _ in range(3))
    p = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    check(u15b200.lib().u15c_thw_indexes(p(ids), len(ids), IMG, CTX, p(g) if len(grids) else None,
                                         len(grids), p(t), p(h), p(w)))
    return t, h, w


def prompt(text_before, grids, text_after):
    ids = list(range(100, 100 + text_before))
    for gh, gw in grids:
        ids += [IMG] + [CTX] * ((gh // 2) * (gw // 2)) + [END]
    ids += list(range(200, 200 + text_after))
    return ids


def test_text_only_is_causal_positions():
    t, h, w = thw(list(range(100, 113)), [])
    assert list(t) == list(range(13)) and not h.any() and not w.any()


def test_one_image_hand_derived():
    # 2 text tokens, <img>, 2x3 context tokens (grid 4 x 6), </img>, 1 text
    ids = prompt(2, [(4, 6)], 1)
    t, h, w = thw(ids, [(4, 6)])
    #        x  x  <img> ctx * 6             </img> x
    assert list(t) == [0, 1, 2] + [3] * 6 + [4, 5]
    assert list(h[3:9]) == [0, 0, 0, 1, 1, 1] and list(w[3:9]) == [0, 1, 2, 0, 1, 2]
    assert not h[:3].any() and not h[9:].any()


@pytest.mark.parametrize("grids", [[(28, 40)], [(28, 40), (16, 16)], [(2, 2), (6, 4), (8, 8)]])
def test_reference_test_properties(grids):
    ids = prompt(7, grids, 5)
    t, h, w = thw(ids, grids)
    ids = np.array(ids)
    ctx = ids == CTX
    # every image's context run shares one t, one above its <img>
    starts = np.where(ids == IMG)[0]
    for k, s in enumerate(starts):
        n = (grids[k][0] // 2) * (grids[k][1] // 2)
        run = t[s + 1:s + 1 + n]
        assert (run == t[s] + 1).all()
        assert list(h[s + 1:s + 1 + n]) == [i // (grids[k][1] // 2) for i in range(n)]
        assert list(w[s + 1:s + 1 + n]) == [i % (grids[k][1] // 2) for i in range(n)]
    # the generated image sits at max(t) + 1, NOT at the token count
    gen_t = int(t.max()) + 1
    assert gen_t < len(ids)
    assert gen_t == len(ids) - ctx.sum() + len(grids)
    assert not h[~ctx].any() and not w[~ctx].any()


def test_matches_restated_rule_on_random_sequences():
    rng = np.random.default_rng(3)
    for _ in range(50):
        grids = [(int(2 * rng.integers(1, 6)), int(2 * rng.integers(1, 6)))
                 for _ in range(rng.integers(0, 4))]
        ids = prompt(int(rng.integers(0, 9)), grids, int(rng.integers(0, 9)))
        got = thw(ids, grids)
        want = O.thw_indexes(ids, IMG, CTX, grids)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)
