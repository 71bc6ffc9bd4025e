"""Seeded synthetic workloads for the voice-detect B200 engine.

The reference ships no model weights and no audio corpus that covers its
benchmark configs, so every parity test and benchmark runs on synthetic inputs
with the shapes and value distributions the benchmark configs name:

* clips   -- 16 kHz mono int16: a sum of 8 harmonics of f0 ~ U(100, 250) Hz with
             seeded amplitudes and phases, plus pink (1/f) noise at -20 dB
             relative to the harmonic RMS, scaled to a -6 dBFS peak. Seed =
             base_seed + clip index. The C ABI takes f32 PCM = int16 / 32768.
* weights -- WeSpeaker ResNet34 topology (stem 1->32; BasicBlock stages [3,4,6,3]
             at 32/64/128/256 channels, stride 2 entering stages 2-4, 1x1
             downsample on every stage entry; TSTP; FC 5120->256), Kaiming-normal
             conv weights with BatchNorm (gamma 1, beta 0, mean ~ N(0, 0.1),
             var ~ U(0.5, 1.5), eps 1e-5) folded into weight + bias, exactly what
             the reference's ONNX-derived GGUFs carry (src/encoder_resnet.cpp:16-20).
* GGUF    -- written with the reference's KV schema (``voicedetect.*``, see
             src/model_loader.cpp:114-215 and the converter's writer), f32, f16 or
             q8_0 weights. q8_0 4-D conv weights are a NEW format (the reference
             never quantises conv weights): they are stored OHWI, i.e. ggml ne =
             [IC, KW, KH, OC], so the 32-element q8_0 blocks run along IC.
"""
from __future__ import annotations

import numpy as np

SR = 16000
N_MELS = 80


# ---------------------------------------------------------------------------
# Clips
# ---------------------------------------------------------------------------
def make_clip(seed: int, n_samples: int) -> np.ndarray:
    """One synthetic int16 clip of n_samples at 16 kHz (see module docstring)."""
    rng = np.random.default_rng(seed)
    f0 = rng.uniform(100.0, 250.0)
    amps = rng.uniform(0.3, 1.0, 8) / np.arange(1, 9)
    phases = rng.uniform(0.0, 2.0 * np.pi, 8)
    t = np.arange(n_samples, dtype=np.float64) / SR
    h = np.zeros(n_samples, np.float64)
    for k in range(8):
        f = f0 * (k + 1)
        if f < SR / 2:
            h += amps[k] * np.sin(2.0 * np.pi * f * t + phases[k])
    white = rng.standard_normal(n_samples)
    spec = np.fft.rfft(white)
    freqs = np.fft.rfftfreq(n_samples, 1.0 / SR)
    shape = np.zeros_like(freqs)
    shape[1:] = 1.0 / np.sqrt(freqs[1:])
    pink = np.fft.irfft(spec * shape, n=n_samples)
    h_rms = np.sqrt(np.mean(h * h)) + 1e-12
    p_rms = np.sqrt(np.mean(pink * pink)) + 1e-12
    x = h + pink * (h_rms * 10.0 ** (-20.0 / 20.0) / p_rms)
    x *= 0.5 / (np.max(np.abs(x)) + 1e-12)  # -6 dBFS peak
    return np.round(x * 32767.0).astype(np.int16)


def clip_f32(clip16: np.ndarray) -> np.ndarray:
    return (clip16.astype(np.float32) / 32768.0).astype(np.float32)


def clip_lengths(seed: int, n: int, lo_s: float = 2.0, hi_s: float = 20.0) -> np.ndarray:
    """Seeded U(lo, hi) s clip lengths in samples (benchmark config 4)."""
    rng = np.random.default_rng(seed)
    return np.round(rng.uniform(lo_s, hi_s, n) * SR).astype(np.int64)


# ---------------------------------------------------------------------------
# ResNet34 weights
# ---------------------------------------------------------------------------
def _folded_conv(rng, oc: int, ic: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    w = rng.standard_normal((oc, ic, k, k)) * np.sqrt(2.0 / (ic * k * k))
    mean = rng.normal(0.0, 0.1, oc)
    var = rng.uniform(0.5, 1.5, oc)
    scale = 1.0 / np.sqrt(var + 1e-5)
    wf = (w * scale[:, None, None, None]).astype(np.float32)
    bf = (-mean * scale).astype(np.float32)
    return wf, bf


def resnet34_model(seed: int = 0, n_mels: int = N_MELS, channels=(32, 64, 128, 256),
                   blocks=(3, 4, 6, 3), emb_dim: int = 256, mean_vec: bool = True) -> dict:
    """Synthetic WeSpeaker ResNet34: dict with torch-order f32 arrays.

    Keys: stem_w (C0,1,3,3), stem_b, blocks[i] = {conv1_w, conv1_b, conv2_w, conv2_b,
    [down_w (OC,IC,1,1), down_b], stride}, seg_w (emb, 2*C*F'), seg_b, mean_vec,
    var_eps, l2_normalize."""
    rng = np.random.default_rng(seed)
    m: dict = {}
    m["stem_w"], m["stem_b"] = _folded_conv(rng, channels[0], 1, 3)
    bl = []
    cin = channels[0]
    f = n_mels
    for si, (c, n) in enumerate(zip(channels, blocks)):
        for bi in range(n):
            stride = 2 if (si > 0 and bi == 0) else 1
            b: dict = {"stride": stride}
            b["conv1_w"], b["conv1_b"] = _folded_conv(rng, c, cin, 3)
            b["conv2_w"], b["conv2_b"] = _folded_conv(rng, c, c, 3)
            if stride != 1 or cin != c:
                b["down_w"], b["down_b"] = _folded_conv(rng, c, cin, 1)
            bl.append(b)
            cin = c
        if si > 0:
            f = (f + 2 - 3) // 2 + 1
    m["blocks"] = bl
    pooled = 2 * cin * f
    m["seg_w"] = (rng.standard_normal((emb_dim, pooled)) / np.sqrt(pooled)).astype(np.float32)
    m["seg_b"] = rng.normal(0.0, 0.01, emb_dim).astype(np.float32)
    m["mean_vec"] = rng.normal(0.0, 0.05, emb_dim).astype(np.float32) if mean_vec else None
    m["var_eps"] = 1e-8
    m["l2_normalize"] = True
    return m


def tiny_resnet_model(seed: int = 0, n_mels: int = 16) -> dict:
    """A small ResNet (same topology rules, narrower/shallower) for fast CPU tests."""
    return resnet34_model(seed, n_mels=n_mels, channels=(32, 64, 128, 256), blocks=(1, 1, 1, 1))


def quantize_q8_0_model(m: dict) -> dict:
    """Round-trip every q8_0-eligible weight through gguf's q8_0 so the oracle sees
    exactly the values a q8_0 GGUF carries. Conv weights are quantised along IC
    (OHWI order); 2-D FC weights along their input dim."""
    import gguf
    from gguf import quants

    q = dict(m)

    def rt_conv(w):
        if w.shape[1] % 32 != 0:
            return w
        ohwi = np.ascontiguousarray(w.transpose(0, 2, 3, 1))
        qb = quants.quantize(ohwi, gguf.GGMLQuantizationType.Q8_0)
        d = quants.dequantize(qb, gguf.GGMLQuantizationType.Q8_0).reshape(ohwi.shape)
        return np.ascontiguousarray(d.transpose(0, 3, 1, 2)).astype(np.float32)

    def rt_2d(w):
        if w.shape[1] % 32 != 0:
            return w
        qb = quants.quantize(np.ascontiguousarray(w), gguf.GGMLQuantizationType.Q8_0)
        return quants.dequantize(qb, gguf.GGMLQuantizationType.Q8_0).reshape(w.shape).astype(
            np.float32)

    q["blocks"] = []
    for b in m["blocks"]:
        nb = dict(b)
        for k in ("conv1_w", "conv2_w", "down_w"):
            if k in b:
                nb[k] = rt_conv(b[k])
        q["blocks"].append(nb)
    q["seg_w"] = rt_2d(m["seg_w"])
    return q


def f16_model(m: dict) -> dict:
    """Round every weight tensor through f16 (what an f16 GGUF carries)."""
    def r(a):
        return None if a is None else a.astype(np.float16).astype(np.float32)
    q = {k: (r(v) if isinstance(v, np.ndarray) else v) for k, v in m.items() if k != "blocks"}
    q["blocks"] = [{k: (r(v) if isinstance(v, np.ndarray) else v) for k, v in b.items()}
                   for b in m["blocks"]]
    return q


# ---------------------------------------------------------------------------
# GGUF writer (reference KV schema)
# ---------------------------------------------------------------------------
def write_resnet_gguf(path: str, m: dict, dtype: str = "f32") -> None:
    """Write a wespeaker_resnet34 GGUF. dtype: f32 | f16 | q8_0 (weights only;
    biases, mean_vec and the IC=1 stem stay f32)."""
    import gguf
    from gguf import quants

    w = gguf.GGUFWriter(path, arch="voicedetect")
    w.add_string("voicedetect.arch", "wespeaker_resnet34")
    w.add_uint32("voicedetect.embedding_dim", int(m["seg_w"].shape[0]))
    w.add_bool("voicedetect.l2_normalize", bool(m.get("l2_normalize", True)))
    w.add_uint32("voicedetect.fbank.sample_rate", 16000)
    w.add_uint32("voicedetect.fbank.n_mels", int(m.get("n_mels", N_MELS)))
    w.add_uint32("voicedetect.fbank.n_fft", 512)
    w.add_uint32("voicedetect.fbank.win_length", 400)
    w.add_uint32("voicedetect.fbank.hop_length", 160)
    w.add_float32("voicedetect.fbank.preemph", 0.97)
    w.add_float32("voicedetect.fbank.low_freq", 20.0)
    w.add_float32("voicedetect.fbank.high_freq", 0.0)
    w.add_bool("voicedetect.fbank.use_energy", False)
    w.add_bool("voicedetect.fbank.cmn", True)
    w.add_string("voicedetect.fbank.window", "povey")

    tensors: list[tuple[str, np.ndarray, str]] = []

    def add(name: str, arr: np.ndarray, kind: str):
        tensors.append((name, arr, kind))
        return name

    add("stem.weight", m["stem_w"], "conv")
    add("stem.bias", m["stem_b"], "bias")
    c1w, c1b, c2w, c2b, dw, db, st = [], [], [], [], [], [], []
    for i, b in enumerate(m["blocks"]):
        c1w.append(add(f"blk{i}.conv1.weight", b["conv1_w"], "conv"))
        c1b.append(add(f"blk{i}.conv1.bias", b["conv1_b"], "bias"))
        c2w.append(add(f"blk{i}.conv2.weight", b["conv2_w"], "conv"))
        c2b.append(add(f"blk{i}.conv2.bias", b["conv2_b"], "bias"))
        if "down_w" in b:
            dw.append(add(f"blk{i}.down.weight", b["down_w"], "conv"))
            db.append(add(f"blk{i}.down.bias", b["down_b"], "bias"))
        else:
            dw.append("")
            db.append("")
        st.append(int(b["stride"]))
    add("seg.weight", m["seg_w"], "fc")
    add("seg.bias", m["seg_b"], "bias")
    if m.get("mean_vec") is not None:
        add("mean_vec", m["mean_vec"], "bias")

    w.add_string("voicedetect.resnet.stem_weight", "stem.weight")
    w.add_string("voicedetect.resnet.stem_bias", "stem.bias")
    w.add_array("voicedetect.resnet.conv1_weight", c1w)
    w.add_array("voicedetect.resnet.conv1_bias", c1b)
    w.add_array("voicedetect.resnet.conv2_weight", c2w)
    w.add_array("voicedetect.resnet.conv2_bias", c2b)
    w.add_array("voicedetect.resnet.down_weight", dw)
    w.add_array("voicedetect.resnet.down_bias", db)
    w.add_array("voicedetect.resnet.stride", st)
    w.add_string("voicedetect.resnet.seg_weight", "seg.weight")
    w.add_string("voicedetect.resnet.seg_bias", "seg.bias")
    w.add_string("voicedetect.resnet.mean_vec", "mean_vec" if m.get("mean_vec") is not None else "")
    w.add_float32("voicedetect.resnet.var_eps", float(m.get("var_eps", 1e-8)))

    for name, arr, kind in tensors:
        arr = np.ascontiguousarray(arr, np.float32)
        if dtype == "f32" or kind == "bias" or (kind == "conv" and arr.shape[1] == 1):
            w.add_tensor(name, arr)
        elif dtype == "f16":
            w.add_tensor(name, arr.astype(np.float16))
        elif dtype == "q8_0":
            if kind == "conv":
                if arr.shape[1] % 32 != 0:
                    w.add_tensor(name, arr)
                    continue
                arr = np.ascontiguousarray(arr.transpose(0, 2, 3, 1))  # OHWI
            elif arr.shape[-1] % 32 != 0:
                w.add_tensor(name, arr)
                continue
            qb = quants.quantize(arr, gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, qb, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            raise ValueError(dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
