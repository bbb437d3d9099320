"""Seeded synthetic weights and inputs in the reference model's on-disk format.

The real parakeet-redux weights are not available, so every workload runs on random-init weights of the exact
architecture (reference/config.json, reference/ternary.json): ternary modules in `thrush-ternary-v2` (5 base-3
digits per byte, least significant digit first, code = trit + 1; crates/voxrt/src/trits.rs:1-41) with f16 scales
per 128 input columns, dense parameters as f32 (f16-rounded where the format stores f16).
"""
from __future__ import annotations

import numpy as np

D_MODEL, FF, HEADS, CONV_K, N_LAYERS, N_MELS, SUB_CH, GROUP = 1024, 4096, 8, 9, 24, 128, 256, 128

_POW3 = np.array([1, 3, 9, 27, 81], dtype=np.uint16)


def pack_trits(trits: np.ndarray) -> np.ndarray:
    """int8 [out, n] in {-1,0,1} -> thrush-ternary-v2 bytes [out, ceil(n/5)] (pad digits 0)."""
    out, n = trits.shape
    rb = (n + 4) // 5
    codes = np.zeros((out, rb * 5), np.uint16)
    codes[:, :n] = (trits.astype(np.int16) + 1).astype(np.uint16)
    return (codes.reshape(out, rb, 5) * _POW3).sum(-1).astype(np.uint8)


def random_trits(rng, out, inp, p=(0.3, 0.4, 0.3)) -> np.ndarray:
    u = rng.random((out, inp), dtype=np.float32)
    return ((u >= p[0]).astype(np.int8) + (u >= p[0] + p[1]).astype(np.int8) - 1).astype(np.int8)


def ternary_module(rng, out, inp, group=GROUP, p=(0.3, 0.4, 0.3), scale_lo=0.01, scale_hi=0.05, trits=None):
    """One ternary module as the model file stores it: qweight u8 [out, ceil(in/5)], scales f16 bits [out, in/g]."""
    if trits is None:
        trits = random_trits(rng, out, inp, p)
    scales = rng.uniform(scale_lo, scale_hi, size=(out, inp // group)).astype(np.float16)
    return {"qweight": pack_trits(trits), "scales": scales.view(np.uint16), "out": out, "in": inp, "group": group}


def stack_modules(mods):
    """TernaryLinear::load_stacked (ternary_linear.rs:59-99): concatenate rows of modules sharing an input."""
    return {"qweight": np.concatenate([m["qweight"] for m in mods]),
            "scales": np.concatenate([m["scales"] for m in mods]),
            "out": sum(m["out"] for m in mods), "in": mods[0]["in"], "group": mods[0]["group"]}


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def layer(seed: int, d=D_MODEL, ff=FF, heads=HEADS, k=CONV_K, group=GROUP):
    """One FastConformer layer (BASELINE config 2 distributions)."""
    rng = np.random.default_rng(seed)
    dh = d // heads
    L = {
        "ff1_1": ternary_module(rng, ff, d, group), "ff1_2": ternary_module(rng, d, ff, group),
        "qkv": stack_modules([ternary_module(rng, d, d, group) for _ in range(3)]),
        "o": ternary_module(rng, d, d, group), "relk": ternary_module(rng, d, d, group),
        "pw1": ternary_module(rng, 2 * d, d, group), "pw2": ternary_module(rng, d, d, group),
        "ff2_1": ternary_module(rng, ff, d, group), "ff2_2": ternary_module(rng, d, ff, group),
    }
    for n in ("norm_ff1", "norm_attn", "norm_conv", "norm_ff2", "norm_out"):
        L[n + "_w"] = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        L[n + "_b"] = (0.1 * rng.standard_normal(d)).astype(np.float32)
    L["bias_u"] = _f16(0.1 * rng.standard_normal((heads, dh)))
    L["bias_v"] = _f16(0.1 * rng.standard_normal((heads, dh)))
    L["dw_weight"] = _f16(0.1 * rng.standard_normal((d, 1, k)))
    L["bn_w"] = _f16(1.0 + 0.1 * rng.standard_normal(d))
    L["bn_b"] = _f16(0.1 * rng.standard_normal(d))
    L["bn_mean"] = _f16(0.1 * rng.standard_normal(d))
    L["bn_var"] = _f16(rng.uniform(0.5, 1.5, d))
    return L


def subsampling(seed: int, c=SUB_CH, n_mels=N_MELS, d=D_MODEL, k=3):
    """dw-striding Conv2d x8 front end, HF tensor layouts (subsampling.rs:31-96), He-scaled, f16-rounded."""
    rng = np.random.default_rng(seed)
    f3 = n_mels // 8
    he = lambda fan_in, shape: _f16(rng.standard_normal(shape) * np.sqrt(2.0 / fan_in))
    return {
        "conv0_w": he(k * k, (c, 1, k, k)), "conv0_b": _f16(0.01 * rng.standard_normal(c)),
        "dw1_w": he(k * k, (c, 1, k, k)), "dw1_b": _f16(0.01 * rng.standard_normal(c)),
        "pw1_w": he(c, (c, c, 1, 1)), "pw1_b": _f16(0.01 * rng.standard_normal(c)),
        "dw2_w": he(k * k, (c, 1, k, k)), "dw2_b": _f16(0.01 * rng.standard_normal(c)),
        "pw2_w": he(c, (c, c, 1, 1)), "pw2_b": _f16(0.01 * rng.standard_normal(c)),
        "lin_w": _f16(rng.standard_normal((d, c * f3)) * np.sqrt(1.0 / (c * f3))),
        "lin_b": _f16(0.01 * rng.standard_normal(d)),
        "n_mels": n_mels,
    }


def encoder(n_layers=N_LAYERS, base_seed=100, sub_seed=99):
    """Full encoder: layer i uses seed base_seed + i."""
    return {"sub": subsampling(sub_seed), "layers": [layer(base_seed + i) for i in range(n_layers)]}


def out_frames(t_in: int, k=3, s=2) -> int:
    """Subsampling::out_frames (subsampling.rs:99-106)."""
    p = (k - 1) // 2
    n = t_in
    for _ in range(3):
        n = (n + 2 * p - k) // s + 1
    return n


def mel_frames(seconds: float, sr=16000, hop=160) -> int:
    """Log-mel frame count for a clip (center-padded STFT, hop 160 at 16 kHz: frontend.rs MelConfig)."""
    return int(round(seconds * sr)) // hop + 1


def feats(rng, t_in: int, n_mels=N_MELS) -> np.ndarray:
    """Stand-in log-mel features [t_in, n_mels]: the frontend normalises every mel bin per utterance to zero mean
    and unit variance, so normalised features are modelled as N(0, 1)."""
    return rng.standard_normal((t_in, n_mels)).astype(np.float32)


def config3_lengths(seed=3, n=64, lo=2.0, hi=30.0):
    """64 utterances, lengths U(2, 30) s."""
    return np.random.default_rng(seed).uniform(lo, hi, n)


def config3_workload(rank=0, n=64):
    """The config-3 batch one GPU rank processes: lengths U(2, 30) s (seeded per rank), their log-mel frame counts
    and stand-in features. Returns (seconds [n], t_in [n] int32, feats list of [t_in, n_mels] f32)."""
    secs = config3_lengths(seed=3 + 1009 * rank, n=n)
    t_in = np.array([mel_frames(s) for s in secs], np.int32)
    rng = np.random.default_rng(300 + rank)
    return secs, t_in, [feats(rng, int(t)) for t in t_in]


def config5_lengths(seed=5, n=4096, lo=1.0, hi=60.0):
    """4096 utterances, lengths log-uniform in [1, 60] s."""
    return np.exp(np.random.default_rng(seed).uniform(np.log(lo), np.log(hi), n))


def decoder(seed=7, hidden=640, vocab=8193, d_model=D_MODEL, n_layers=2, durations=(0, 1, 2, 3, 4), max_symbols=10):
    """Random-init TDT decoder of the reference's shapes (LSTM 640 x 2, joint 640, vocab 8193
    with blank = 8192, durations 0-4, at most 10 symbols per frame). PyTorch default inits: embedding N(0, 1),
    LSTM / linear weights and biases U(-1/sqrt(fan_in), 1/sqrt(fan_in)); the tensors the model file stores as f16
    (LSTM, decoder projector, joint head) are f16 bit patterns."""
    rng = np.random.default_rng(seed)
    u = lambda shape, fan: rng.uniform(-1.0, 1.0, shape) / np.sqrt(fan)
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16).view(np.uint16)
    n_out = vocab + len(durations)
    return {
        "hidden": hidden, "vocab": vocab, "blank": vocab - 1, "durations": list(durations),
        "max_symbols": max_symbols, "d_model": d_model,
        "embedding": rng.standard_normal((vocab, hidden)).astype(np.float32),
        "lstm": [{"w_ih": f16(u((4 * hidden, hidden), hidden)), "w_hh": f16(u((4 * hidden, hidden), hidden)),
                  "b_ih": u(4 * hidden, hidden).astype(np.float32), "b_hh": u(4 * hidden, hidden).astype(np.float32)}
                 for _ in range(n_layers)],
        "proj_w": f16(u((hidden, hidden), hidden)), "proj_b": u(hidden, hidden).astype(np.float32),
        "head_w": f16(u((n_out, hidden), hidden)), "head_b": u(n_out, hidden).astype(np.float32),
        "enc_w": u((hidden, d_model), d_model).astype(np.float32), "enc_b": u(hidden, d_model).astype(np.float32),
    }


# ------------------------------------------------------------------------------------- model directories
_ST_DTYPE = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.uint8): "U8",
             np.dtype(np.int8): "I8"}


def vad_weights(tensors: dict) -> dict:
    """The VAD head's weights (f32, from the f16 tensors of `model_dir_tensors`) as VadHead and the oracle take them."""
    g = lambda n: np.asarray(tensors["vad_head." + n], np.float32)
    return {"proj_w": g("proj.weight"), "proj_b": g("proj.bias"), "ctx_w": g("ctx.weight"), "ctx_b": g("ctx.bias"),
            "out_w": g("out.weight"), "out_b": float(g("out.bias")[0])}


def write_safetensors(path, tensors: dict):
    """A safetensors file: u64 little-endian header length, the JSON header (name -> dtype, shape, data_offsets,
    padded with spaces to a multiple of 8 bytes), then the tensors' bytes in header order."""
    import json

    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": _ST_DTYPE[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def model_dir_tensors(enc: dict, dec: dict, vad_hidden=128, vad_kernel=5, seed=11):
    """The tensors of a thrush-ternary-v2 model file for a synthetic encoder (`encoder()`) and decoder
    (`decoder()`), named and typed as the reference's loaders read them (format.rs:153-309). Tensors the format
    stores as f16 are rounded to f16; returns (tensors, quantized-module specs)."""
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16)
    t, qm = {}, []

    def tern(name, m):
        t[name + ".qweight"] = np.asarray(m["qweight"], np.uint8)
        t[name + ".scales"] = np.asarray(m["scales"]).view(np.float16)
        qm.append({"name": name, "out_features": m["out"], "in_features": m["in"], "group_size": m["group"],
                   "as_conv1d": "pointwise" in name, "has_bias": False, "zero_fraction": 0.4})

    s = enc["sub"]
    for idx, k in ((0, "conv0"), (2, "dw1"), (3, "pw1"), (5, "dw2"), (6, "pw2")):
        t[f"encoder.subsampling.layers.{idx}.weight"] = f16(s[k + "_w"])
        t[f"encoder.subsampling.layers.{idx}.bias"] = np.asarray(s[k + "_b"], np.float32)
    t["encoder.subsampling.linear.weight"] = f16(s["lin_w"])
    t["encoder.subsampling.linear.bias"] = np.asarray(s["lin_b"], np.float32)
    for i, L in enumerate(enc["layers"]):
        p = f"encoder.layers.{i}"
        d = L["qkv"]["out"] // 3
        qkv = {k: L["qkv"][k] for k in ("qweight", "scales")}
        for j, n in enumerate(("q_proj", "k_proj", "v_proj")):
            tern(f"{p}.self_attn.{n}", {"qweight": qkv["qweight"][j * d:(j + 1) * d],
                                        "scales": qkv["scales"][j * d:(j + 1) * d], "out": d,
                                        "in": L["qkv"]["in"], "group": L["qkv"]["group"]})
        for n, k in (("feed_forward1.linear1", "ff1_1"), ("feed_forward1.linear2", "ff1_2"), ("self_attn.o_proj", "o"),
                     ("self_attn.relative_k_proj", "relk"), ("conv.pointwise_conv1", "pw1"),
                     ("conv.pointwise_conv2", "pw2"), ("feed_forward2.linear1", "ff2_1"),
                     ("feed_forward2.linear2", "ff2_2")):
            tern(f"{p}.{n}", L[k])
        for n, k in (("norm_feed_forward1", "norm_ff1"), ("norm_self_att", "norm_attn"), ("norm_conv", "norm_conv"),
                     ("norm_feed_forward2", "norm_ff2"), ("norm_out", "norm_out")):
            t[f"{p}.{n}.weight"] = np.asarray(L[k + "_w"], np.float32)
            t[f"{p}.{n}.bias"] = np.asarray(L[k + "_b"], np.float32)
        t[f"{p}.conv.norm.weight"] = np.asarray(L["bn_w"], np.float32)
        t[f"{p}.conv.norm.bias"] = np.asarray(L["bn_b"], np.float32)
        t[f"{p}.conv.norm.running_mean"] = np.asarray(L["bn_mean"], np.float32)
        t[f"{p}.conv.norm.running_var"] = np.asarray(L["bn_var"], np.float32)
        t[f"{p}.conv.depthwise_conv.weight"] = f16(L["dw_weight"])
        t[f"{p}.self_attn.bias_u"] = f16(L["bias_u"])
        t[f"{p}.self_attn.bias_v"] = f16(L["bias_v"])
    t["encoder_projector.weight"] = f16(dec["enc_w"])
    t["encoder_projector.bias"] = np.asarray(dec["enc_b"], np.float32)
    t["decoder.embedding.weight"] = f16(dec["embedding"])
    for l, L in enumerate(dec["lstm"]):
        t[f"decoder.lstm.weight_ih_l{l}"] = np.asarray(L["w_ih"]).view(np.float16)
        t[f"decoder.lstm.weight_hh_l{l}"] = np.asarray(L["w_hh"]).view(np.float16)
        t[f"decoder.lstm.bias_ih_l{l}"] = np.asarray(L["b_ih"], np.float32)
        t[f"decoder.lstm.bias_hh_l{l}"] = np.asarray(L["b_hh"], np.float32)
    t["decoder.decoder_projector.weight"] = np.asarray(dec["proj_w"]).view(np.float16)
    t["decoder.decoder_projector.bias"] = np.asarray(dec["proj_b"], np.float32)
    t["joint.head.weight"] = np.asarray(dec["head_w"]).view(np.float16)
    t["joint.head.bias"] = np.asarray(dec["head_b"], np.float32)
    rng = np.random.default_rng(seed)
    dm = enc["layers"][0]["qkv"]["in"]
    t["vad_head.proj.weight"] = f16(0.02 * rng.standard_normal((vad_hidden, dm, 1)))
    t["vad_head.proj.bias"] = f16(0.02 * rng.standard_normal(vad_hidden))
    t["vad_head.ctx.weight"] = f16(0.05 * rng.standard_normal((vad_hidden, vad_hidden, vad_kernel)))
    t["vad_head.ctx.bias"] = f16(0.02 * rng.standard_normal(vad_hidden))
    t["vad_head.out.weight"] = f16(0.1 * rng.standard_normal((1, vad_hidden, 1)))
    t["vad_head.out.bias"] = f16(0.02 * rng.standard_normal(1))
    return t, qm


def write_model_dir(path, enc: dict, dec: dict, tensors=None, qm=None, fmt="thrush-ternary-v2",
                    vad_hidden=128, vad_kernel=5):
    """Write a model directory in the reference's layout (config.json, ternary.json, model.safetensors) for the
    synthetic encoder / decoder; `tensors` / `qm` override the generated ones (tests that corrupt a file)."""
    import json
    import os

    os.makedirs(path, exist_ok=True)
    if tensors is None:
        tensors, qm = model_dir_tensors(enc, dec, vad_hidden, vad_kernel)
    L0, s = enc["layers"][0], enc["sub"]
    d, heads = L0["qkv"]["in"], np.asarray(L0["bias_u"]).shape[0]
    cfg = {
        "encoder_config": {"hidden_size": d, "intermediate_size": L0["ff1_1"]["out"],
                           "num_hidden_layers": len(enc["layers"]), "num_attention_heads": heads,
                           "num_mel_bins": int(s["n_mels"]), "conv_kernel_size": np.asarray(L0["dw_weight"]).shape[-1],
                           "subsampling_conv_channels": np.asarray(s["conv0_w"]).shape[0],
                           "subsampling_conv_kernel_size": np.asarray(s["conv0_w"]).shape[-1],
                           "subsampling_conv_stride": 2, "subsampling_factor": 8, "max_position_embeddings": 5000,
                           "scale_input": False},
        "blank_token_id": dec["blank"], "decoder_hidden_size": dec["hidden"], "num_decoder_layers": len(dec["lstm"]),
        "durations": list(dec["durations"]), "max_symbols_per_step": dec["max_symbols"], "vocab_size": dec["vocab"],
        "ternary_group_size": L0["qkv"]["group"], "ternary_modules": [m["name"] for m in qm],
    }
    tern = {"format": fmt, "names": "hf",
            "vad_head": {"d_model": d, "hidden": vad_hidden, "kernel": vad_kernel, "frame_seconds": 0.08},
            "quantized_modules": qm, "n_quantized_params": int(sum(m["out_features"] * m["in_features"] for m in qm)),
            "n_dense_params": 0}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    with open(os.path.join(path, "ternary.json"), "w") as f:
        json.dump(tern, f)
    write_safetensors(os.path.join(path, "model.safetensors"), tensors)
    return path


def decoder_f16_rounded(dec: dict) -> dict:
    """The decoder dict with the tensors a model file stores as f16 (embedding, encoder projector) rounded to f16,
    i.e. the values a decoder loaded from `write_model_dir` sees."""
    r = dict(dec)
    r["embedding"] = np.asarray(dec["embedding"], np.float32).astype(np.float16).astype(np.float32)
    r["enc_w"] = np.asarray(dec["enc_w"], np.float32).astype(np.float16).astype(np.float32)
    return r


def bandlimited_noise(rng, seconds: float, sr=16000, lo=100.0, hi=7000.0, dbfs=-20.0) -> np.ndarray:
    """BASELINE config 3's synthetic audio: white Gaussian noise through a fixed 4th-order Butterworth band-pass
    (100-7000 Hz), scaled to the given RMS level in dBFS. f32 samples."""
    from scipy.signal import butter, sosfilt

    n = int(round(seconds * sr))
    sos = butter(4, [lo, hi], btype="bandpass", fs=sr, output="sos")
    y = sosfilt(sos, rng.standard_normal(n))
    rms = float(np.sqrt(np.mean(y * y))) if n else 1.0
    return (y * (10.0 ** (dbfs / 20.0) / max(rms, 1e-12))).astype(np.float32)
