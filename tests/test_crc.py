"""CRC-32C of expert packs (the checked layer loads): the oracle's bitwise definition is
pinned to published check values, and the library's host CRC matches it (no GPU)."""
import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

# Published CRC-32C check values: the CRC catalogue's "123456789" check, and the iSCSI
# test patterns of RFC 3720 (appendix B.4), 32 bytes each.
KNOWN = [
    (b"123456789", 0xE3069283),
    (bytes(32), 0x8A9136AA),
    (b"\xff" * 32, 0x62A8AB43),
    (bytes(range(32)), 0x46DD794E),
    (bytes(range(31, -1, -1)), 0x113FDB5C),
    (b"", 0x00000000),
]


@pytest.mark.parametrize("data,want", KNOWN)
def test_oracle_known_values(data, want):
    assert O.crc32c(data) == want


@pytest.mark.parametrize("data,want", KNOWN)
def test_library_known_values(data, want):
    assert N.crc32c(data) == want


@pytest.mark.parametrize("n", [1, 7, 8, 9, 63, 64, 4095, 4096, 100003])
def test_library_matches_oracle(n):
    a = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8)
    assert N.crc32c(a) == O.crc32c(a)


def test_continuation_and_combine():
    a = np.random.default_rng(1).integers(0, 256, 10000, dtype=np.uint8)
    whole = N.crc32c(a)
    for cut in (0, 1, 8, 4097, 9999):
        assert N.crc32c(a[cut:], N.crc32c(a[:cut])) == whole
        assert N.lib().nmoe_crc32c_combine(N.crc32c(a[:cut]), N.crc32c(a[cut:]), a.size - cut) == whole


def test_expert_crcs_of_an_image():
    lw = O.make_layer(3, bits=4, num_experts=4)
    crcs = N.expert_crcs(lw.experts, 4)
    esz = N.expert_size(4)
    assert crcs.shape == (4,)
    for i in range(4):
        assert crcs[i] == O.crc32c(lw.experts.view(np.uint8)[i * esz:(i + 1) * esz])
