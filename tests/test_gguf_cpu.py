"""CPU: the GGUF reader of the library (s2k_gguf_read_hparams,
s2k_gguf_tensor_info) on files written by gguf-py's GGUFWriter with the
reference's keys and tensor names: the hyper-parameters equal the model's,
and every tensor's name, type, shape, data offset and size equal what
gguf-py's own GGUFReader reports.  No device is needed."""
from __future__ import annotations

import os

import numpy as np
import pytest

import s2k
import synthetic
from gguf_fixture import write_model_gguf

gguf = pytest.importorskip("gguf")


@pytest.mark.parametrize("quant", ["q8_0", "q4_k_m", "f16"])
def test_gguf_hparams_and_tensor_directory(tmp_path, quant):
    hp = synthetic.preset("small")
    tensors = list(synthetic.make_model(hp, seed=2, quant=quant, norm_std=0.1))
    path = os.path.join(tmp_path, f"small_{quant}.gguf")
    write_model_gguf(path, hp, tensors)
    got = s2k.gguf_read_hparams(path)
    for name in synthetic.FIELDS:
        want = getattr(hp, name)
        assert got[name] == pytest.approx(want), name
    ours = s2k.gguf_tensors(path)
    theirs = gguf.GGUFReader(path).tensors
    assert len(ours) == len(theirs) == len(tensors) + 1
    by_name = {spec.name: (spec, buf) for spec, buf in tensors}
    for (name, t, ne, off, nb), rt in zip(ours, theirs):
        assert name == rt.name
        assert t == int(rt.tensor_type)
        assert ne[: len(rt.shape)] == tuple(int(x) for x in rt.shape)
        assert off == int(rt.data_offset)
        assert nb == int(rt.n_bytes)
        if name in by_name:
            spec, buf = by_name[name]
            assert (t, ne[0], ne[1]) == (spec.type, spec.ne0, spec.ne1)
            with open(path, "rb") as fh:
                fh.seek(off)
                assert fh.read(nb) == np.asarray(buf).tobytes()


def test_gguf_defaults_and_rejects(tmp_path):
    path = os.path.join(tmp_path, "bare.gguf")
    w = gguf.GGUFWriter(path, arch="fish-speech")
    w.add_uint32("fish-speech.block_count", 3)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    hp = s2k.gguf_read_hparams(path)
    # missing keys take load_shared's defaults (src/s2_model.cpp:258-287)
    assert hp["block_count"] == 3 and hp["vocab_size"] == 155776 and hp["semantic_begin_id"] == 151678
    assert hp["has_fast_decoder"] == 1 and hp["fast_block_count"] == 4 and hp["attention_qk_norm"] == 0
    bad = os.path.join(tmp_path, "bad.gguf")
    with open(bad, "wb") as fh:
        fh.write(b"GGML" + bytes(20))
    with pytest.raises(s2k.S2KError) as e:
        s2k.gguf_read_hparams(bad)
    assert e.value.status == -1
    trunc = os.path.join(tmp_path, "trunc.gguf")
    hp_small = synthetic.preset("small")
    write_model_gguf(trunc, hp_small, list(synthetic.make_model(hp_small, seed=2)))
    data = open(trunc, "rb").read()
    with open(trunc, "wb") as fh:
        fh.write(data[: len(data) // 2])
    with pytest.raises(s2k.S2KError):
        s2k.gguf_read_hparams(trunc)
