"""The stream-K work split of the pair GEMM (SegWalk in sam3cpp_b200/csrc/gemm.cu),
restated here to check its invariants for many shapes on CPU: every (tile,
K block) unit is computed exactly once; a tile is shared by at most two
neighbouring pairs; the pair holding a tile's first K blocks (kSegOut) walks
that segment first, and the next pair walks the tile's remaining K blocks
(kSegIn) last, so the hand-over can never wait in a cycle; and the
launcher's enabling rule (at least as many tiles as pairs) keeps every range
at least one tile long."""

import itertools

import pytest

FULL, OUT, IN = 0, 1, 2


def seg_walk(pair, n_pairs, n_tiles, num_kb, sk):
    """The segments (tile, k0, k1, role) of one CTA pair, in walk order."""
    if not sk:
        return [(t, 0, num_kb, FULL) for t in range(pair, n_tiles, n_pairs)]
    units = n_tiles * num_kb
    u0, u1 = units * pair // n_pairs, units * (pair + 1) // n_pairs
    segs = []
    if u1 % num_kb:
        segs.append((u1 // num_kb, 0, u1 % num_kb, OUT))
    segs += [(t, 0, num_kb, FULL) for t in range(-(-u0 // num_kb), u1 // num_kb)]
    if u0 % num_kb:
        segs.append((u0 // num_kb, u0 % num_kb, num_kb, IN))
    return segs


def check_plan(n_tiles, num_kb, n_pairs, sk):
    walks = [seg_walk(p, n_pairs, n_tiles, num_kb, sk) for p in range(n_pairs)]
    covered = {}
    for p, segs in enumerate(walks):
        for t, k0, k1, role in segs:
            assert 0 <= t < n_tiles and 0 <= k0 < k1 <= num_kb
            for k in range(k0, k1):
                assert (t, k) not in covered, (t, k)
                covered[(t, k)] = p
    assert len(covered) == n_tiles * num_kb
    for p, segs in enumerate(walks):
        roles = [s[3] for s in segs]
        assert roles.count(OUT) <= 1 and roles.count(IN) <= 1
        if OUT in roles:
            assert roles[0] == OUT                      # the head first
            t, _, k1, _ = segs[0]
            nxt = walks[p + 1]
            assert nxt[-1] == (t, k1, num_kb, IN)       # the next pair takes the tail, last
        if IN in roles:
            assert roles[-1] == IN
            t, k0, _, _ = segs[-1]
            assert walks[p - 1][0] == (t, 0, k0, OUT)
    return walks


@pytest.mark.parametrize("n_pairs", [74, 72, 70, 66, 37])
@pytest.mark.parametrize("num_kb", [5, 8, 16, 74])
def test_stream_k_covers_every_unit_once(n_pairs, num_kb):
    # the launcher enables stream-K only with at least as many tiles as pairs
    for n_tiles in itertools.chain(range(n_pairs, n_pairs + 40), [84, 164, 252, 324, 399]):
        if n_tiles >= n_pairs:
            check_plan(n_tiles, num_kb, n_pairs, True)


def test_whole_tiles_cover_every_unit_once():
    for n_tiles, n_pairs in [(1, 74), (84, 74), (5184, 74), (3, 2)]:
        check_plan(n_tiles, 8, min(n_pairs, n_tiles), False)


def test_one_image_fc2_plan():
    """fc2 at one image: 84 tiles of 74 K blocks on 74 pairs, 84 units each."""
    walks = check_plan(84, 74, 74, True)
    assert walks[0] == [(1, 0, 10, OUT), (0, 0, 74, FULL)]
    assert walks[1] == [(2, 0, 20, OUT), (1, 10, 74, IN)]
    assert sum(k1 - k0 for t, k0, k1, _ in walks[40]) == 84
