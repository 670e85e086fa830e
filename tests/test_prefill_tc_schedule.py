"""Host restatement of the tcgen05 prefill kernel's schedule and hand-off protocol (CPU).

`pythonintern_b200/csrc/prefill_tc.cu` pairs adjacent Q tiles of a sequence into work
items and runs a producer lane, an MMA-issuing warp and two groups of four softmax warps
that hand tiles to each other through mbarriers.  These tests restate both in Python:

* the item enumeration (``count_pairs`` / ``find_item``) covers every (sequence, Q tile,
  kv head) exactly once, and each tile's K/V tile count reaches its last position;
* the barrier protocol (phases, parities, buffer indices as the kernel computes them)
  finishes under random completion orders of the asynchronous operations, and no buffer
  is rewritten before its reader is done: the S buffer before the softmax read it, P
  before the PV MMA consumed it (P lives over its S buffer), O before the epilogue read
  it, a Q buffer before the last S MMA of its item.  TMA copies land in any order; the
  MMA warp's commits arrive in issue order (a tcgen05.commit fires once every earlier
  tcgen05 operation of its thread has completed), which is what lets a softmax warp that
  has seen S(n) complete rely on PV(n - 2) having landed, so that a parity wait on the
  PV barrier never sees a phase two behind.
"""

import random

import pytest

KT, NG, ST, GW = 64, 2, 3, 4


def items(lens, ctx0, qt, nkv):
    """The kernel's work items in order: (seq, kv head, [(t0, nt, n_kv)] * 2)."""
    out = []
    for s, L in enumerate(lens):
        ntile = (L + qt - 1) // qt if L > 0 else 0
        for u in range((ntile + 1) // 2):
            tiles = []
            for q in range(NG):
                tile = 2 * u + q  # counted from the end of the sequence
                if tile < ntile:
                    t0 = (ntile - 1 - tile) * qt
                    nt = min(qt, L - t0)
                    tiles.append((t0, nt, (ctx0[s] + t0 + nt - 1) // KT + 1))
                else:
                    tiles.append((0, 0, 0))
            for g in range(nkv):
                out.append((s, g, tiles))
    # item w = kv head w % nkv of pair w / nkv: regroup pair-major
    by_pair = {}
    for s, g, tiles in out:
        by_pair.setdefault((s, tuple(tiles)), []).append((s, g, tiles))
    return [it for grp in by_pair.values() for it in grp]


@pytest.mark.parametrize("qt", [16, 32, 64, 128])
def test_items_cover_every_tile_once(qt):
    rnd = random.Random(qt)
    for _ in range(20):
        n = rnd.randint(1, 9)
        lens = [rnd.randint(0, 700) for _ in range(n)]
        ctx0 = [rnd.choice([0, 0, rnd.randint(0, 300)]) for _ in range(n)]
        nkv = rnd.choice([1, 2, 8])
        seen = {}
        for s, g, tiles in items(lens, ctx0, qt, nkv):
            assert tiles[0][1] > 0  # the later tile of a pair always exists
            assert tiles[1][2] <= tiles[0][2]  # the earlier tile needs no more K/V tiles
            for t0, nt, n_kv in tiles:
                if nt == 0:
                    continue
                key = (s, g, t0)
                assert key not in seen
                seen[key] = nt
                last_pos = ctx0[s] + t0 + nt - 1
                assert n_kv * KT > last_pos >= (n_kv - 1) * KT
        want = {(s, g, t * qt) for s, L in enumerate(lens) for g in range(nkv)
                for t in range((L + qt - 1) // qt)}
        assert set(seen) == want
        assert sum(seen.values()) == sum(lens) * nkv


class Bar:
    def __init__(self, count):
        self.count, self.arrived, self.done = count, 0, 0

    def arrive(self):
        self.arrived += 1
        if self.arrived == self.count:
            self.arrived, self.done = 0, self.done + 1

    def ready(self, parity):  # mbarrier.try_wait.parity
        return (self.done & 1) != parity


def simulate(work, seed):
    """Producer, MMA warp and NG x GW softmax warps as coroutines over the kernel's barriers;
    TMA copies land in a random order, the MMA warp's commits in issue order.  Returns
    True when every role finished."""
    rnd = random.Random(seed)
    q_full = [[Bar(1), Bar(1)] for _ in range(NG)]
    q_empty = [[Bar(1), Bar(1)] for _ in range(NG)]
    kv_full, kv_empty = [Bar(1) for _ in range(ST)], [Bar(1) for _ in range(ST)]
    s_full = [[Bar(1), Bar(1)] for _ in range(NG)]
    p_full = [[Bar(GW), Bar(GW)] for _ in range(NG)]
    pv_done = [[Bar(1), Bar(1)] for _ in range(NG)]
    o_empty = [Bar(GW) for _ in range(NG)]
    pending = []  # TMA completions, any order
    commits = []  # tcgen05.commit arrivals, in issue order
    s_read = [[0] * GW for _ in range(NG)]      # S tiles read, per softmax warp
    p_written = [[0] * GW for _ in range(NG)]   # P tiles written
    o_read = [[0] * GW for _ in range(NG)]      # items whose O was read out
    pv_issued, pv_landed = [0] * NG, [0] * NG

    def producer():
        iq, J = [0, 0], 0
        for tiles in work:
            for g in range(NG):
                if tiles[g][1] == 0:
                    continue
                qb = iq[g] & 1
                while not q_empty[g][qb].ready(((iq[g] >> 1) & 1) ^ 1):
                    yield
                pending.append((q_full[g][qb], None))
                iq[g] += 1
            for _ in range(tiles[0][2]):
                st = J % ST
                while not kv_empty[st].ready(((J // ST) & 1) ^ 1):
                    yield
                pending.append((kv_full[st], None))
                J += 1

    def mma():
        iq, js, jp, io, qb, J = [0, 0], [0, 0], [0, 0], [0, 0], [0, 0], 0

        def issue_pv(g, first):
            pb = jp[g] & 1
            while not p_full[g][pb].ready((jp[g] >> 1) & 1):
                yield
            if first:
                while not o_empty[g].ready((io[g] & 1) ^ 1):
                    yield
                assert min(o_read[g]) >= io[g], "O overwritten before the epilogue read it"
                io[g] += 1
            assert min(p_written[g]) > jp[g], "PV issued before its P"
            pv_issued[g] += 1
            commits.append((pv_done[g][pb], g))
            jp[g] += 1

        for tiles in work:
            n_kv = [t[2] for t in tiles]
            for g in range(NG):
                if tiles[g][1] == 0:
                    continue
                qb[g] = iq[g] & 1
                while not q_full[g][qb[g]].ready((iq[g] >> 1) & 1):
                    yield
                iq[g] += 1
            for j in range(n_kv[0]):
                st = J % ST
                while not kv_full[st].ready((J // ST) & 1):
                    yield
                for g in range(NG):
                    if j >= n_kv[g]:
                        continue
                    # S(n) into buffer n & 1: its previous reader (S(n - 2)) is done
                    assert min(s_read[g]) >= js[g] - 1, "S rewritten before it was read"
                    # P(n - 2), which lives over that buffer, has been consumed: PV(n - 2)
                    # was issued before, and the tensor cores run in issue order
                    assert pv_issued[g] >= js[g] - 1
                    commits.append((s_full[g][js[g] & 1], None))
                    js[g] += 1
                    if j == n_kv[g] - 1:
                        commits.append((q_empty[g][qb[g]], None))
                if j >= 1:
                    for g in range(NG):
                        if j - 1 < n_kv[g]:
                            yield from issue_pv(g, j == 1)
                    commits.append((kv_empty[(J - 1) % ST], None))
                J += 1
            for g in range(NG):
                if n_kv[g] == n_kv[0] and n_kv[0] > 0:
                    yield from issue_pv(g, n_kv[0] == 1)
            commits.append((kv_empty[(J - 1) % ST], None))

    def softmax(grp, wid):
        js = 0
        for tiles in work:
            if tiles[grp][1] == 0:
                continue
            for j in range(tiles[grp][2]):
                b = js & 1
                while not s_full[grp][b].ready((js >> 1) & 1):
                    yield
                s_read[grp][wid] = js + 1
                if j >= 1 and rnd.random() < 0.3:  # a rescale of O needs PV(js - 1) landed
                    while not pv_done[grp][(js - 1) & 1].ready(((js - 1) >> 1) & 1):
                        yield
                    assert pv_landed[grp] >= js
                p_written[grp][wid] = js + 1
                p_full[grp][b].arrive()
                js += 1
            while not pv_done[grp][(js - 1) & 1].ready(((js - 1) >> 1) & 1):
                yield
            assert pv_landed[grp] >= js, "epilogue before the item's last PV landed"
            o_read[grp][wid] += 1
            o_empty[grp].arrive()

    roles = [producer(), mma()] + [softmax(g, w) for g in range(NG) for w in range(GW)]
    alive = list(range(len(roles)))
    for _ in range(3_000_000):
        if not alive:
            return True
        if pending and rnd.random() < 0.3:
            pending.pop(rnd.randrange(len(pending)))[0].arrive()
        if commits and rnd.random() < 0.3:
            bar, g = commits.pop(0)
            if g is not None:
                pv_landed[g] += 1
            bar.arrive()
        r = rnd.choice(alive)
        try:
            next(roles[r])
        except StopIteration:
            alive.remove(r)
    return False


@pytest.mark.parametrize("qt", [16, 32, 128])
@pytest.mark.parametrize("lens,ctx0", [([1], [0]), ([5, 130, 77], [0, 17, 0]), ([300, 1, 64, 65], [200, 0, 0, 9])])
def test_protocol_finishes_without_early_reuse(qt, lens, ctx0):
    work = [tiles for _, _, tiles in items(lens, ctx0, qt, 1)]
    for seed in range(2):
        assert simulate(work, seed)
