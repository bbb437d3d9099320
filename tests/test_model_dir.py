"""CPU: the thrush-ternary-v2 model-directory loader (ModelFile, crates/voxrt/src/format.rs:76-309) on synthetic
model directories written in the reference's layout: open, validate, config, tensor access, exact f16 -> f32
widening, the reference's rejection cases, and the TDT decoder loaded from the directory agreeing bit for bit with
the one built from the same arrays."""
import json
import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    from voxrt_b200 import synth

    enc = synth.encoder(2)
    dec = synth.decoder(seed=7)
    path = str(tmp_path_factory.mktemp("model") / "m")
    tensors, qm = synth.model_dir_tensors(enc, dec)
    synth.write_model_dir(path, enc, dec, tensors=tensors, qm=qm)
    return path, enc, dec, tensors, qm


def _rewrite(tmp_path, enc, dec, tensors, qm, **kw):
    from voxrt_b200 import synth

    p = str(tmp_path / "bad")
    synth.write_model_dir(p, enc, dec, tensors=tensors, qm=qm, **kw)
    return p


def test_open_validate_config(small_model):
    from voxrt_b200.model import ModelFile

    path, enc, dec, tensors, qm = small_model
    m = ModelFile.open(path)
    assert m.validate() == []
    c = m.config()
    assert (c["d_model"], c["ff"], c["n_layers"], c["heads"], c["n_mels"], c["conv_kernel"]) == (1024, 4096, 2, 8, 128, 9)
    assert (c["dec_hidden"], c["dec_layers"], c["vocab"], c["blank"], c["max_symbols"], c["n_durations"]) == \
        (640, 2, 8193, 8192, 10, 5)
    assert (c["vad_hidden"], c["vad_kernel"], c["vad_frame_seconds"]) == (128, 5, 0.08)
    q = m.tensor("encoder.layers.1.self_attn.k_proj.qweight")
    np.testing.assert_array_equal(q, tensors["encoder.layers.1.self_attn.k_proj.qweight"])
    w = m.tensor_f32("encoder.subsampling.linear.weight")
    np.testing.assert_array_equal(w, tensors["encoder.subsampling.linear.weight"].astype(np.float32))
    m.close()


def test_f16_widening_is_exact_for_every_pattern(tmp_path, small_model):
    """Every one of the 65,536 f16 bit patterns (subnormals, infinities and NaNs included) widens as numpy does."""
    from voxrt_b200 import synth
    from voxrt_b200.model import ModelFile

    path, enc, dec, tensors, qm = small_model
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    t2 = dict(tensors)
    t2["extra.all_f16"] = allh.reshape(256, 256)
    p = _rewrite(tmp_path, enc, dec, t2, qm)
    m = ModelFile.open(p)
    got = m.tensor_f32("extra.all_f16").ravel()
    want = allh.astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    m.close()


def test_rejections(tmp_path, small_model):
    """ModelFile::open refuses another format or naming; validate lists missing tensors, wrong dtypes / shapes and a
    dense .weight beside a qweight (format.rs:94-106, 153-309)."""
    from voxrt_b200._lib import VxgError
    from voxrt_b200.model import ModelFile

    path, enc, dec, tensors, qm = small_model
    with pytest.raises(VxgError, match="unsupported format"):
        ModelFile.open(_rewrite(tmp_path / "f", enc, dec, tensors, qm, fmt="thrush-ternary-v1"))
    t = dict(tensors)
    del t["encoder.layers.0.norm_out.bias"]
    t["encoder.layers.1.conv.depthwise_conv.weight"] = t["encoder.layers.1.conv.depthwise_conv.weight"].astype(np.float32)
    t["joint.head.bias"] = t["joint.head.bias"][:-1]
    t["encoder.layers.0.self_attn.o_proj.weight"] = np.zeros((4, 4), np.float16)
    m = ModelFile.open(_rewrite(tmp_path / "v", enc, dec, t, qm))
    probs = m.validate()
    assert "missing encoder.layers.0.norm_out.bias" in probs
    assert any(p.startswith("encoder.layers.1.conv.depthwise_conv.weight: got F32") for p in probs)
    assert any(p.startswith("joint.head.bias: got F32 [8197]") for p in probs)
    assert "encoder.layers.0.self_attn.o_proj.weight present alongside qweight" in probs
    assert len(probs) == 4
    m.close()
    # a truncated safetensors file is refused at open
    p = _rewrite(tmp_path / "t", enc, dec, tensors, qm)
    st = os.path.join(p, "model.safetensors")
    with open(st, "r+b") as f:
        f.truncate(os.path.getsize(st) - 1000)
    with pytest.raises(VxgError, match="data offsets"):
        ModelFile.open(p)
    # broken JSON
    with open(os.path.join(p, "ternary.json"), "w") as f:
        f.write('{"format": "thrush-ternary-v2", "names": ')
    with pytest.raises(VxgError, match="ternary.json"):
        ModelFile.open(p)


def test_decoder_from_model_matches_arrays(small_model):
    """Decoder::load from the directory == the decoder built from the same (f16-rounded) arrays: LSTM step, joint
    and greedy emissions, bit for bit (host)."""
    from voxrt_b200 import synth
    from voxrt_b200.decoder import TdtDecoder

    path, enc, dec, tensors, qm = small_model
    a = TdtDecoder(synth.decoder_f16_rounded(dec))
    b = TdtDecoder.from_model(path)
    rng = np.random.default_rng(3)
    h = rng.standard_normal((2, 640)).astype(np.float32)
    c = rng.standard_normal((2, 640)).astype(np.float32)
    for x, y in zip(a.pred_step(17, h, c), b.pred_step(17, h, c)):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    e = rng.standard_normal(640).astype(np.float32)
    assert np.array_equal(a.joint(e, h[0]).view(np.uint32), b.joint(e, h[0]).view(np.uint32))
    proj = rng.standard_normal((40, 640)).astype(np.float32)
    np.testing.assert_array_equal(a.greedy(proj), b.greedy(proj))
    a.close()
    b.close()
