"""C ABI surface checks that need no GPU: the library loads, exports every symbol the
header declares, and its host-only helpers (pack layout, layout.json validation,
argument checks) behave like the reference's pack contract."""
import json
import os
import re

import numpy as np
import pytest

import nmoe_b200 as N
from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "nmoe", "moe_cuda.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nmoe_(?:moe|lm_head|linear_attn|full_attn|decoder)_\w+|nmoe_crc32c\w*)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = N.lib()
    names = header_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(N.ABI_SYMBOLS)


@pytest.mark.parametrize("bits", [4, 2])
def test_expert_size_and_offsets_match_pack_format(bits):
    assert N.expert_size(bits) == O.expert_size(bits)
    assert N.expert_offsets(bits) == O.expert_offsets(bits)
    meta = json.load(open(os.path.join(REPO, "tests", "golden", "golden_meta.json")))["blobs"][f"q{bits}"]
    assert N.expert_offsets(bits) == [o for _, o, _ in meta["layout"]]
    assert N.expert_size(bits) == meta["size"]
    assert N.expert_size(3) == 0


def converter_layout(bits):
    """layout.json exactly as scripts/convert_qwen36.py:351-359 writes it."""
    meta = json.load(open(os.path.join(REPO, "tests", "golden", "golden_meta.json")))["blobs"][f"q{bits}"]
    return {"expert_size": meta["size"], "num_layers": 40, "num_experts": 256,
            "components": [{"name": n, "offset": o, "size": s} for n, o, s in meta["layout"]]}


@pytest.mark.parametrize("bits", [4, 2])
def test_validate_layout_json_accepts_converter_output(tmp_path, bits):
    p = tmp_path / "layout.json"
    p.write_text(json.dumps(converter_layout(bits), indent=2))
    assert N.validate_layout_json(str(p), bits) == (N.OK, "")
    # the other bit width must be rejected
    rc, msg = N.validate_layout_json(str(p), 6 - bits)
    assert rc == N.ESIZE and "expert_size" in msg


def test_validate_layout_json_rejects_bad_files(tmp_path):
    p = tmp_path / "layout.json"
    good = converter_layout(4)
    cases = []
    bad = json.loads(json.dumps(good)); bad["components"][3]["offset"] += 4; cases.append((bad, "offset/size"))
    bad = json.loads(json.dumps(good)); bad["components"][0]["name"] = "up_proj.weight"; cases.append((bad, "unexpected"))
    bad = json.loads(json.dumps(good)); del bad["components"][8]; cases.append((bad, "9 entries"))
    bad = json.loads(json.dumps(good)); del bad["expert_size"]; cases.append((bad, "expert_size"))
    bad = json.loads(json.dumps(good)); bad["components"][0]["dtype"] = "u16"; cases.append((bad, "dtype"))
    bad = json.loads(json.dumps(good)); bad["components"][0]["shape"] = [512, 128]; cases.append((bad, "shape"))
    bad = json.loads(json.dumps(good)); bad["bits"] = 2; cases.append((bad, "bits"))
    for obj, frag in cases:
        p.write_text(json.dumps(obj))
        rc, msg = N.validate_layout_json(str(p), 4)
        assert rc == N.ESIZE and frag in msg, (frag, rc, msg)
    # optional reference-style keys that agree are accepted
    ok = json.loads(json.dumps(good))
    ok["bits"] = 4
    ok["components"][0].update({"dtype": "U32", "shape": [512, 256]})
    p.write_text(json.dumps(ok))
    assert N.validate_layout_json(str(p), 4)[0] == N.OK
    p.write_text("{not json")
    assert N.validate_layout_json(str(p), 4)[0] == N.ESIZE
    assert N.validate_layout_json(str(tmp_path / "missing.json"), 4)[0] == N.EIO


def test_create_rejects_bad_config_without_touching_a_gpu():
    for kw in ({"quant_bits": 3}, {"k_max": 0}, {"k_max": 9}, {"num_layers": 0}, {"num_experts": 300},
               {"router_dtype": N.DTYPE_F32}, {"world_size": 2, "rank": 2}, {"world_size": 3, "rank": 0}):
        with pytest.raises(N.NmoeError) as ei:
            N.Context(**kw)
        assert ei.value.status == N.EINVAL, kw


def test_strerror():
    L = N.lib()
    assert L.nmoe_moe_strerror(N.OK) == b"ok"
    assert b"timed out" in L.nmoe_moe_strerror(N.ETIMEOUT)


def test_timeline_summary_decodes_stamps():
    """summarize_timeline: microseconds after the earliest CTA start, per named phase,
    ignoring unreached slots and surviving a wrap of the 32-bit stamp words."""
    base = 2**32 - 150    # the low word wraps between the CTAs' starts
    tl = np.zeros((3, 16), np.uint32)
    for c in range(3):
        tl[c, 0] = (base + 100 * (2 - c)) & 0xFFFFFFFF
        tl[c, 7] = (base + 20000 + 1000 * c) & 0xFFFFFFFF   # earliest start is CTA 2
    tl[1, 11] = (base + 9000) & 0xFFFFFFFF
    s = N.summarize_timeline(tl)
    assert s["end"] == (20.0, 21.0, 22.0)
    assert s["first unit landed"] == (9.0, 9.0, 9.0)
    assert "act staged" not in s
