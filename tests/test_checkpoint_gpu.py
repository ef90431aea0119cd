"""Checkpoints (zilla_net_save / zilla_net_load, GPU): the SafeTensors F32
layout of the reference's ModelSerializer (param_i in parameter order, compact
JSON header padded with spaces to 8 bytes), read and written here by a
restatement of the format (SafeTensorsSerializer::save/load,
src/Serialization/SafeTensorsSerializer.php:32-98,118-178).
"""
import json
import os
import struct

import numpy as np
import pytest

from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import LM, Net

pytestmark = pytest.mark.gpu


def st_read(path):
    raw = open(path, "rb").read()
    hs = struct.unpack("<Q", raw[:8])[0]
    hdr_bytes = raw[8:8 + hs]
    hdr = json.loads(hdr_bytes)
    meta = hdr.pop("__metadata__", None)
    data = {k: (v["shape"], np.frombuffer(raw[8 + hs + v["data_offsets"][0]:8 + hs + v["data_offsets"][1]], "<f4"))
            for k, v in hdr.items()}
    return hdr_bytes, hdr, data, meta


def st_write(path, tensors):
    """tensors: list of (name, shape, float32 array), in order (as the reference writes them)."""
    header, off, blob = {}, 0, b""
    for name, shape, arr in tensors:
        b = np.ascontiguousarray(arr, "<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": list(shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blob += b
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + blob)


def cnn_shapes(w):
    out = []
    c, h, wd = w.in_shape
    for kind, a, b, p in w.layers:
        if kind == configs.CONV:
            out += [[b, a, 3, 3], [b]]
            c, h, wd = b, h + 2 * p - 2, wd + 2 * p - 2
        elif kind == configs.LINEAR:
            out += [[a, b], [b]]
    return out


def test_save_load_roundtrip_with_adam_state(tmp_path):
    w = configs.CNN_LARGE
    batches = [synthetic.batch(w, 64, seed=9, step=s) for s in range(3)]
    a = Net(w, batch=64, precision=1)
    b = Net(w, batch=64, precision=1)
    try:
        a.set_params(synthetic.init_params(w, seed=9))
        a.step_host(*batches[0])
        a.step_host(*batches[1])
        path = str(tmp_path / "ckpt.safetensors")
        a._check(a.lib.zilla_net_save(a.id, path.encode(), 1))
        # layout: param_i, adam_m_i, adam_v_i with the parameter shapes, compact header
        hdr_bytes, hdr, data, meta = st_read(path)
        shapes = cnn_shapes(w)
        names = [f"param_{i}" for i in range(len(shapes))]
        names += [f"adam_m_{i}" for i in range(len(shapes))] + [f"adam_v_{i}" for i in range(len(shapes))]
        assert list(hdr.keys()) == names
        assert all(hdr[f"param_{i}"]["shape"] == s for i, s in enumerate(shapes))
        assert len(hdr_bytes) % 8 == 0 and meta == {"adam_t": "2"}
        expect = dict(hdr)
        expect["__metadata__"] = meta
        assert hdr_bytes.rstrip(b" ") == json.dumps(expect, separators=(",", ":")).encode()
        p = a.params()
        flat = np.concatenate([data[f"param_{i}"][1] for i in range(len(shapes))])
        assert np.array_equal(flat, p)
        # a fresh net resumes exactly: one more step on each ends bit-identical
        b.set_params(synthetic.init_params(w, seed=1))
        b._check(b.lib.zilla_net_load(b.id, path.encode()))
        assert np.array_equal(b.params(), p)
        la = a.step_host(*batches[2])
        lb = b.step_host(*batches[2])
        assert la == lb
        assert np.array_equal(a.params(), b.params()), "Adam state not restored"
    finally:
        a.close()
        b.close()


def test_load_reference_layout_and_rejects(tmp_path):
    w = configs.WORKLOADS["cnn_1x8_pool_fc"]
    net = Net(w, batch=64, precision=0)
    try:
        shapes = cnn_shapes(w)
        rng = np.random.default_rng(3)
        arrays = [rng.standard_normal(int(np.prod(s))).astype(np.float32) for s in shapes]
        good = str(tmp_path / "ref.safetensors")
        st_write(good, [(f"param_{i}", s, x) for i, (s, x) in enumerate(zip(shapes, arrays))])
        net._check(net.lib.zilla_net_load(net.id, good.encode()))
        assert np.array_equal(net.params(), np.concatenate(arrays))
        bad_shape = str(tmp_path / "bad_shape.safetensors")
        st_write(bad_shape, [(f"param_{i}", (s[::-1] if i == 0 else s), x)
                             for i, (s, x) in enumerate(zip(shapes, arrays))])
        missing = str(tmp_path / "missing.safetensors")
        st_write(missing, [(f"param_{i}", s, x) for i, (s, x) in enumerate(zip(shapes, arrays)) if i != 1])
        truncated = str(tmp_path / "truncated.safetensors")
        open(truncated, "wb").write(open(good, "rb").read()[:-8])
        for path in (bad_shape, missing, truncated, str(tmp_path / "absent.safetensors")):
            assert net.lib.zilla_net_load(net.id, path.encode()) == -2, path
        assert np.array_equal(net.params(), np.concatenate(arrays)), "a rejected load changed the parameters"
    finally:
        net.close()


def test_lm_save_load(tmp_path):
    w = configs.TRANSFORMER_LM
    a = LM(w, batch=4, seq=32)
    b = LM(w, batch=4, seq=32)
    try:
        a.set_params(synthetic.lm_init_params(w, seed=2))
        path = str(tmp_path / "lm.safetensors")
        a._check(a.lib.zilla_net_save(a.id, path.encode(), 0))
        _, hdr, data, meta = st_read(path)
        assert meta is None and hdr["param_0"]["shape"] == [w.vocab, w.dim]
        b._check(b.lib.zilla_net_load(b.id, path.encode()))
        assert np.array_equal(a.params(), b.params())
    finally:
        a.close()
        b.close()
