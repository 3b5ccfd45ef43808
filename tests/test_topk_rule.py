"""The selection scheme of the device top-k (warp_topk_lane, csrc/nmoe_topk.cuh), modelled
on the host and checked against the reference's rule (nmoe_cpu_topk, src/math.m:95-132:
descending, lower index first on ties).

The device scheme: lane l holds experts 8l..8l+7 as order-preserving integer keys
(-0 and +0 share a key) and sorts them once, stably; each round takes the warp maximum
of the lanes' heads, and the lowest lane holding it pops its head. The model below runs
the same steps on the same keys. The adversarial inputs put many exact ties inside a
lane and across lanes, and include infinities and signed zeros."""
import numpy as np
import pytest

from oracle import oracle as O


def order_key(v: np.ndarray) -> np.ndarray:
    u = (np.asarray(v, np.float32) + np.float32(0.0)).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)


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
    v = np.asarray(logits, np.float32)
    order = sorted(range(v.size), key=lambda i: (-float(v[i]), i))
    return np.array(order[:k], np.uint32)


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
