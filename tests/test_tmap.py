"""The tensor-map table the attention template declares for the runtime (CPU only): its
records match the kernel's tile geometry, and no emitted load uses cluster multicast."""

import re

import pytest

from emmyptx.lower import tmap
from emmyptx.lower.attention import BKV_FOR_D


def _table(ptx):
    m = re.search(r"emmy_tmap_desc\[(\d+)\] = \{([^}]*)\};", ptx)
    assert m, "attention PTX declares emmy_tmap_desc"
    words = [int(w) for w in m.group(2).split(",")]
    assert len(words) == int(m.group(1))
    return words


def _records(words):
    assert words[0] == tmap.TMAP_MAGIC
    n = words[1]
    assert len(words) == 2 + n * tmap.TMAP_WORDS
    out = []
    for k in range(n):
        w = words[2 + k * tmap.TMAP_WORDS: 2 + (k + 1) * tmap.TMAP_WORDS]
        rank = w[1]
        out.append({
            "param": w[0], "rank": rank, "dims": w[2:2 + rank],
            "strides": [w[7 + 2 * i] | (w[8 + 2 * i] << 32) for i in range(rank - 1)],
            "box": w[15:15 + rank], "swizzle": w[20], "dtype": w[21]})
    return out


@pytest.mark.parametrize("name,D", [("attention_d64", 64), ("attention_d128", 128)])
def test_attention_declares_kt_and_v_maps(name, D):
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    payload, meta = workloads.WORKLOADS[name]()
    ptx, used, _ = compile_payload(payload, meta)
    assert used == "attention"
    k = meta["kernels"][0]
    order = [a["name"] for a in k["args"]]
    shape = {a["name"]: a["shape"] for a in k["args"]}
    B, H, _, S = shape["kt"]
    kt, v = _records(_table(ptx))
    assert kt["param"] == order.index("kt") and v["param"] == order.index("v")
    assert kt["dims"] == [S, D, B * H] and kt["box"] == [32, D, 1]
    assert kt["strides"] == [S * 4, D * S * 4]
    bkv = BKV_FOR_D[D]
    assert v["dims"] == [D, S, B * H] and v["box"] == [32, bkv, 1]
    assert v["strides"] == [D * 4, S * D * 4]
    for r in (kt, v):
        assert r["swizzle"] == tmap.SWIZZLE_128B_ATOM_32B and r["dtype"] == tmap.DTYPE_FLOAT32
        assert r["box"][0] * 4 == 128       # one box row = one 128-byte swizzle row
    # kt copies at two sites (an item's first block, then each next one), a box per 32 keys;
    # v: a box per 32 columns
    assert ptx.count("cp.async.bulk.tensor.3d") == 2 * (bkv // 32) + D // 32
    assert "multicast" not in ptx
    assert "emmy_tmap_key" in ptx and "fence.proxy.tensormap::generic.acquire" in ptx


def test_no_emitted_load_uses_cluster_multicast():
    """No kernel of any benchmark workload names multicast at all (TMA loads, bulk copies and
    tcgen05.commit alike): each CTA loads its own tiles."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    for name, make in workloads.WORKLOADS.items():
        payload, meta = make()
        assert "multicast" not in compile_payload(payload, meta)[0], name


@pytest.mark.parametrize("kw,msg", [
    (dict(dims=[8, 8], strides=[], box=[8, 8]), "disagree"),
    (dict(dims=[8, 8], strides=[36], box=[8, 8]), "multiples of 16"),
    (dict(dims=[8, 8], strides=[32], box=[8, 300]), "within 1..256"),
])
def test_record_rejects_bad_geometry(kw, msg):
    with pytest.raises(ValueError, match=msg):
        tmap.record(0, **kw)
