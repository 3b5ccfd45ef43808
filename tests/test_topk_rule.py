"""The selection scheme of the device top-k (warp_topk_lane, csrc/nmoe_topk.cuh), modelled
on the host and checked against the reference's rule (nmoe_cpu_topk, src/math.m:95-132:
descending, lower index first on ties).

Near ties: the reference selects on its fp32 probabilities p = fl(expf(l - max)) * fl(1/sum),
and two distinct logits one float apart can round to the same p; the reference then puts
the lower id first, the device (which selects on the logits) the larger logit. Whether a
pair collides depends on the platform's expf and on the width of long double in the sum,
so the library defines the ids by the logit rule and the tests check the exact statement:
both rules pick the same sequence of reference probabilities. NaN logits rank below
every other logit on the device; the reference's softmax turns one NaN logit into NaN
probabilities everywhere (its sum is NaN), so NaN inputs are compared with the rule only.

The device scheme: lane l holds experts 8l..8l+7 as order-preserving integer keys
(-0 and +0 share a key) and sorts them once, stably; each round takes the warp maximum
of the lanes' heads, and the lowest lane holding it pops its head. The model below runs
the same steps on the same keys. The adversarial inputs put many exact ties inside a
lane and across lanes, and include infinities and signed zeros."""
import numpy as np
import pytest

from oracle import oracle as O


def order_key(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, np.float32)
    u = (v + np.float32(0.0)).view(np.uint32)
    key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
    return np.where(np.isnan(v), np.uint32(1), key).astype(np.uint32)


def device_scheme(logits: np.ndarray, k: int):
    keys = order_key(logits)
    lanes = []
    for lane in range(32):
        ids = list(range(8 * lane, 8 * lane + 8))
        lanes.append(sorted(ids, key=lambda i: -int(keys[i])))   # stable: ties keep lower id first
    out = []
    for _ in range(k):
        heads = [int(keys[l[0]]) if l else 0 for l in lanes]
        m = max(heads)
        w = heads.index(m)                                            # lowest lane holding the max
        out.append(lanes[w].pop(0))
    return np.array(out, np.uint32)


def rule(logits: np.ndarray, k: int):
    """Descending logits, lower id first on ties, NaN after everything else."""
    v = np.asarray(logits, np.float32)
    order = sorted(range(v.size), key=lambda i: (bool(np.isnan(v[i])), 0.0 if np.isnan(v[i]) else -float(v[i]), i))
    return np.array(order[:k], np.uint32)


def reference_probs(logits: np.ndarray) -> np.ndarray:
    """The reference's fp32 softmax (nmoe_cpu_softmax restated in the oracle)."""
    p = np.array(logits, np.float32, copy=True)
    O.lib().orc_softmax(p, p.size)
    return p


def adjacent_pair_logits(hi_id: int, lo_id: int) -> np.ndarray:
    """All logits 0 except two adjacent floats in [0.25, 0.5) (spacing 2^-25): the larger
    one at hi_id. exp(-2^-25) = 1 - 2^-25 + 2^-51 rounds to 1.0f, so both get the same
    reference probability."""
    v = np.zeros(256, np.float32)
    v[hi_id] = np.float32(0.25) + np.float32(3 * 2.0 ** -25)
    v[lo_id] = np.float32(0.25) + np.float32(2 * 2.0 ** -25)
    assert np.nextafter(v[lo_id], np.float32(1)) == v[hi_id]
    return v


def cases():
    rng = np.random.default_rng(5)
    yield rng.standard_normal(256).astype(np.float32)
    yield np.zeros(256, np.float32)                                   # every logit tied
    yield rng.integers(-3, 4, 256).astype(np.float32)                 # heavy ties everywhere
    v = rng.standard_normal(256).astype(np.float32)
    v[[3, 5, 200, 201, 37]] = 9.0                                     # ties inside and across lanes
    yield v
    v = rng.standard_normal(256).astype(np.float32)
    v[[10, 250]] = np.inf
    v[[0, 1, 2]] = -np.inf
    yield v
    v = np.full(256, -np.inf, np.float32)
    v[[7, 100]] = [0.0, -0.0]                                         # signed zeros compare equal
    yield v
    v = rng.standard_normal(256).astype(np.float32)
    v[8 * 17: 8 * 17 + 8] = 5.0                                       # one lane holds all winners
    yield v
    v = rng.standard_normal(256).astype(np.float32)
    v[[0, 9, 77, 255]] = np.nan                                       # NaN ranks last
    yield v
    v = np.full(256, np.nan, np.float32)
    v[[40, 3]] = [1.0, 2.0]                                           # fewer non-NaN than k
    yield v
    yield adjacent_pair_logits(10, 3)


@pytest.mark.parametrize("k", [1, 2, 3, 8])
def test_device_scheme_matches_reference_rule(k):
    for v in cases():
        np.testing.assert_array_equal(device_scheme(v, k), rule(v, k))


@pytest.mark.parametrize("k", [1, 4, 8])
def test_rule_matches_reference_code_on_integer_logits(k):
    """On logits one apart (distinct probabilities) the reference's own softmax + top-k
    code picks the same experts as the rule, ties included."""
    rng = np.random.default_rng(11)
    for _ in range(5):
        v = rng.integers(-4, 5, 256).astype(np.float32)
        idx, _ = O.route_reference(v, k)
        np.testing.assert_array_equal(idx, rule(v, k))
        np.testing.assert_array_equal(device_scheme(v, k), idx)


@pytest.mark.parametrize("k", [1, 2, 8])
def test_near_tie_same_probability_sequence(k):
    """Adjacent-float logits (ids 10 > 3 by logit) collide in the reference's softmax:
    the device keeps logit order, the reference puts id 3 first; both pick the same
    sequence of reference probabilities."""
    v = adjacent_pair_logits(10, 3)
    p = reference_probs(v)
    assert p[3] == p[10]                       # the collision this case is built for
    ours = device_scheme(v, k)
    assert ours[0] == 10
    ridx, _ = O.route_reference(v, k)
    assert ridx[0] == 3
    np.testing.assert_array_equal(p[ours], p[ridx])
    assert sorted(ours[:2].tolist()) == sorted(ridx[:2].tolist()) or k == 1


def test_random_near_ties_same_probability_sequence():
    """Logit vectors with many adjacent-float pairs around the top-k boundary: wherever
    the two rules order ids differently, the reference probabilities are equal."""
    rng = np.random.default_rng(21)
    collisions = 0
    for _ in range(300):
        v = (rng.standard_normal(256) * 0.3).astype(np.float32)
        top = np.argsort(-v)[:9]
        for a, b in zip(top[::2], top[1::2]):
            v[b] = np.nextafter(v[a], np.float32(-np.inf))
        for k in (4, 8):
            ours = device_scheme(v, k)
            np.testing.assert_array_equal(ours, rule(v, k))
            ridx, _ = O.route_reference(v, k)
            p = reference_probs(v)
            np.testing.assert_array_equal(p[ours], p[ridx])
            collisions += int(not np.array_equal(ours, ridx))
    assert collisions > 0                      # the collision path was exercised


def test_nan_logits_rank_last():
    v = np.random.default_rng(3).standard_normal(256).astype(np.float32)
    v[[5, 130]] = np.nan
    for k in (1, 8):
        ours = device_scheme(v, k)
        assert 5 not in ours and 130 not in ours
        w = np.where(np.isnan(v), np.float32(-np.inf), v)
        ridx, _ = O.route_reference(w, k)
        np.testing.assert_array_equal(ours, ridx)
