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
# ERes2Net weights
# ---------------------------------------------------------------------------
def eres2net_model(seed: int = 0, n_mels: int = N_MELS, m_channels: int = 32,
                   num_blocks=(3, 4, 6, 3), base_width: int = 32, scale: int = 2,
                   emb_dim: int = 512, calibrate: bool = True) -> dict:
    """Synthetic 3D-Speaker ERes2Net with BatchNorm folded into every conv, as a
    flat conv list in the reference's forward-EXECUTION order
    (src/encoder_eres2net.cpp:147-226; manifest src/model_loader.hpp:68-80):

      stem 3x3 1->M (+b, ReLU)
      layer1..layer4 of Res2Net blocks (expansion 2), each block:
        conv1 1x1 (block stride) in->w*scale, then per chunk i: [AFF la1, la2 when
        i > 0 and the layer fuses with AFF] conv3x3 w->w, then conv3 1x1
        w*scale->2P, then the 1x1 shortcut (block stride) when shape changes
      after layer2: layer1_downsample 3x3 s2 (no bias) + AFF(o2, .)
      after layer3: layer2_downsample + AFF; after layer4: layer3_downsample + AFF
    AFF(C): la1 1x1 2C->C/4 (+b) -> SiLU -> la2 1x1 C/4->C (+b) -> tanh.
    Layers 3 and 4 fuse their chunks with AFF, layers 1 and 2 add them.

    calibrate=True (default) replaces the random BatchNorm statistics by the
    statistics of each conv's actual output on a seeded calibration input, in
    execution order, as a trained model's running statistics are (gamma 1, beta
    N(0, 0.1)). With random statistics the 96-conv network is chaotic: rounding
    its activations to f16 alone moves the embedding to cosine ~0.9994 against
    f32, so no f16 implementation could meet a 0.9999 parity gate on it."""
    rng = np.random.default_rng(seed)
    convs: list[dict] = []

    def conv(ic, oc, k, stride=1, bias=True):
        w, b = _folded_conv(rng, oc, ic, k)
        convs.append({"w": w, "b": b if bias else None, "stride": stride})

    def aff(c):
        conv(2 * c, c // 4, 1)
        conv(c // 4, c, 1)

    conv(1, m_channels, 3)  # stem
    in_planes = m_channels
    f = n_mels
    planes_list = [m_channels, 2 * m_channels, 4 * m_channels, 8 * m_channels]
    for li, (planes, n) in enumerate(zip(planes_list, num_blocks)):
        is_aff = li >= 2
        for bi in range(n):
            stride = 2 if (li > 0 and bi == 0) else 1
            width = int(np.floor(planes * base_width / 64.0))
            conv(in_planes, width * scale, 1, stride)
            for i in range(scale):
                if i > 0 and is_aff:
                    aff(width)
                conv(width, width, 3)
            conv(width * scale, 2 * planes, 1)
            if stride != 1 or in_planes != 2 * planes:
                conv(in_planes, 2 * planes, 1, stride)
            in_planes = 2 * planes
        if li > 0:
            f = (f + 2 - 3) // 2 + 1
            # cross-stage fusion after layers 2, 3, 4: downsample the previous fused
            # feature (3x3 s2, BN-less) and AFF it into this layer's output
            conv(planes, 2 * planes, 3, 2, bias=False)
            aff(2 * planes)
    c_last = 2 * planes_list[-1]
    pooled = 2 * c_last * f
    m = {
        "arch": "eres2net", "convs": convs, "m_channels": m_channels, "scale": scale,
        "num_blocks": list(num_blocks), "relu_clamp": 20.0, "var_eps": 1e-8,
        "seg_w": (rng.standard_normal((emb_dim, pooled)) / np.sqrt(pooled)).astype(np.float32),
        "seg_b": rng.normal(0.0, 0.01, emb_dim).astype(np.float32),
        "l2_normalize": True, "n_mels": n_mels,
    }
    if calibrate:
        _calibrate_eres2net(m, np.random.default_rng(seed + 7919))
    return m


def _calibrate_eres2net(m: dict, rng, frames: int = 200) -> None:
    """Re-fold every biased conv of `m` in place with BatchNorm statistics measured
    on its own output: walks the ERes2Net forward (src/encoder_eres2net.cpp:111-226)
    in float64 on a seeded N(0, 2^2) feature map, and for conv i (weights already
    holding the random init) sets w <- w / sqrt(var + 1e-5), b <- beta - mean /
    sqrt(var + 1e-5) from the per-channel mean / variance of w * x over all output
    positions, beta ~ N(0, 0.1). BN-less convs (the cross-stage downsamples) keep
    their weights."""
    import torch
    import torch.nn.functional as Fn

    convs = m["convs"]
    it = iter(range(len(convs)))
    hi = float(m["relu_clamp"])
    S = int(m["scale"])
    M = int(m["m_channels"])
    nb = m["num_blocks"]

    def conv(x):
        c = convs[next(it)]
        w = torch.from_numpy(c["w"].astype(np.float64))
        k = w.shape[-1]
        y = Fn.conv2d(x, w, stride=c["stride"], padding=(k - 1) // 2)
        if c["b"] is None:
            return y
        mu = y.mean((0, 2, 3))
        sc = 1.0 / torch.sqrt(y.var((0, 2, 3)) + 1e-5)
        beta = torch.from_numpy(rng.normal(0.0, 0.1, y.shape[1]))
        c["w"] = (w * sc.view(-1, 1, 1, 1)).numpy().astype(np.float32)
        c["b"] = (beta - mu * sc).numpy().astype(np.float32)
        return (y - mu.view(1, -1, 1, 1)) * sc.view(1, -1, 1, 1) + beta.view(1, -1, 1, 1)

    def aff(x, ds):
        z = Fn.silu(conv(torch.cat([x, ds], 1)))
        return (x + ds) + torch.tanh(conv(z)) * (x - ds)

    in_planes = [M]

    def block(x, planes, is_aff, stride):
        out = conv(x).clamp(0, hi)
        w = out.shape[1] // S
        sp, acc = None, []
        for i in range(S):
            ch = out[:, i * w:(i + 1) * w]
            cur = ch if i == 0 else (aff(sp, ch) if is_aff else sp + ch)
            sp = conv(cur).clamp(0, hi)
            acc.append(sp)
        o = conv(torch.cat(acc, 1))
        res = conv(x) if (stride != 1 or in_planes[0] != 2 * planes) else x
        in_planes[0] = 2 * planes
        return (o + res).clamp(0, hi)

    def layer(x, planes, n, is_aff, stride):
        for b in range(n):
            x = block(x, planes, is_aff, stride if b == 0 else 1)
        return x

    with torch.no_grad():
        feats = torch.from_numpy(rng.standard_normal((1, 1, int(m["n_mels"]), frames)) * 2.0)
        h = torch.relu(conv(feats))
        o1 = layer(h, M, nb[0], False, 1)
        o2 = layer(o1, 2 * M, nb[1], False, 2)
        f12 = aff(o2, conv(o1))
        o3 = layer(o2, 4 * M, nb[2], True, 2)
        f123 = aff(o3, conv(f12))
        o4 = layer(o3, 8 * M, nb[3], True, 2)
        aff(o4, conv(f123))
    assert next(it, None) is None, "calibration walk did not use every conv"


def tiny_eres2net_model(seed: int = 0, n_mels: int = 16) -> dict:
    """Same topology rules, one block per layer and a short front, for CPU tests."""
    return eres2net_model(seed, n_mels=n_mels, num_blocks=(1, 1, 2, 1))


def quantize_model_f16(m: dict) -> dict:
    """Round every ERes2Net weight (not the biases) through f16."""
    q = dict(m)
    q["convs"] = [dict(c, w=c["w"].astype(np.float16).astype(np.float32)) for c in m["convs"]]
    q["seg_w"] = m["seg_w"].astype(np.float16).astype(np.float32)
    return q


def write_eres2net_gguf(path: str, m: dict, dtype: str = "f32") -> None:
    """Write an eres2net GGUF with the reference's KV schema
    (voicedetect.eres2net.*, src/model_loader.cpp:153-165). dtype: f32 | f16
    (weights only; biases and the IC=1 stem stay f32)."""
    import gguf

    w = gguf.GGUFWriter(path, arch="voicedetect")
    w.add_string("voicedetect.arch", "eres2net")
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
    w.add_bool("voicedetect.fbank.cmn", True)
    wn, bn, st = [], [], []
    tensors = []
    for i, c in enumerate(m["convs"]):
        wn.append(f"conv{i}.weight")
        tensors.append((wn[-1], c["w"], "conv"))
        if c["b"] is not None:
            bn.append(f"conv{i}.bias")
            tensors.append((bn[-1], c["b"], "bias"))
        else:
            bn.append("")
        st.append(int(c["stride"]))
    w.add_array("voicedetect.eres2net.conv_weight", wn)
    w.add_array("voicedetect.eres2net.conv_bias", bn)
    w.add_array("voicedetect.eres2net.conv_stride", st)
    w.add_array("voicedetect.eres2net.num_blocks", [int(v) for v in m["num_blocks"]])
    w.add_uint32("voicedetect.eres2net.m_channels", int(m["m_channels"]))
    w.add_uint32("voicedetect.eres2net.scale", int(m["scale"]))
    w.add_string("voicedetect.eres2net.seg_weight", "seg.weight")
    w.add_string("voicedetect.eres2net.seg_bias", "seg.bias")
    w.add_float32("voicedetect.eres2net.relu_clamp", float(m["relu_clamp"]))
    w.add_float32("voicedetect.eres2net.var_eps", float(m["var_eps"]))
    tensors.append(("seg.weight", m["seg_w"], "fc"))
    tensors.append(("seg.bias", m["seg_b"], "bias"))
    for name, arr, kind in tensors:
        arr = np.ascontiguousarray(arr, np.float32)
        if dtype == "f16" and kind != "bias" and not (kind == "conv" and arr.shape[1] == 1
                                                       and arr.shape[2] == 3):
            w.add_tensor(name, arr.astype(np.float16))
        else:
            w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


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


# ---------------------------------------------------------------------------
# ECAPA-TDNN (SpeechBrain layout, the reference's primary arch)
# ---------------------------------------------------------------------------
def ecapa_model(seed: int = 0, n_mels: int = N_MELS, channels: int = 1024, n_blocks: int = 3,
                scale: int = 8, se_channels: int = 128, mfa_channels: int = 1536,
                att_channels: int = 128, emb_dim: int = 192, calibrate: bool = True) -> dict:
    """Synthetic SpeechBrain ECAPA-TDNN as a state dict with the verbatim tensor
    names the reference reads (src/encoder.cpp:157-351, converter
    scripts/convert_voicedetect_to_gguf.py):

      blocks.0                      TDNNBlock k=5: Conv1d n_mels->C, ReLU, BatchNorm1d
      blocks.i (i = 1..n_blocks)    SE-Res2Net: tdnn1 (1x1), res2net_block.blocks.j
                                    (k=3, dilation i+1, C/scale channels, j < scale-1),
                                    tdnn2 (1x1), se_block.conv1/conv2 (1x1, no BN)
      mfa                           TDNNBlock 1x1 n_blocks*C -> mfa_channels
      asp.tdnn / asp.conv           attention: 3*mfa -> att (TDNN), att -> mfa (Conv1d)
      asp_bn.norm                   BatchNorm1d over 2*mfa
      fc.conv                       Conv1d 1x1 2*mfa -> emb_dim

    Conv weights are Kaiming-normal (std sqrt(2 / (IC*k))), biases N(0, 0.05),
    BatchNorm gamma U(0.8, 1.2), beta N(0, 0.1). calibrate=True sets every
    running mean / variance to the statistics of that BatchNorm's input on a
    seeded calibration batch (a trained model's running statistics), like the
    ERes2Net generator; without it the deep random network's activations drift
    far from unit scale."""
    rng = np.random.default_rng(seed)
    sd: dict[str, np.ndarray] = {}

    def conv(name, oc, ic, k):
        sd[name + ".weight"] = (rng.standard_normal((oc, ic, k)) *
                                np.sqrt(2.0 / (ic * k))).astype(np.float32)
        sd[name + ".bias"] = rng.normal(0.0, 0.05, oc).astype(np.float32)

    def bn(name, c):
        sd[name + ".weight"] = rng.uniform(0.8, 1.2, c).astype(np.float32)
        sd[name + ".bias"] = rng.normal(0.0, 0.1, c).astype(np.float32)
        sd[name + ".running_mean"] = rng.normal(0.0, 0.1, c).astype(np.float32)
        sd[name + ".running_var"] = rng.uniform(0.5, 1.5, c).astype(np.float32)

    def tdnn(p, oc, ic, k):
        conv(p + ".conv.conv", oc, ic, k)
        bn(p + ".norm.norm", oc)

    C = channels
    w = C // scale
    tdnn("blocks.0", C, n_mels, 5)
    for i in range(1, n_blocks + 1):
        p = f"blocks.{i}"
        tdnn(p + ".tdnn1", C, C, 1)
        for j in range(scale - 1):
            tdnn(f"{p}.res2net_block.blocks.{j}", w, w, 3)
        tdnn(p + ".tdnn2", C, C, 1)
        conv(p + ".se_block.conv1.conv", se_channels, C, 1)
        conv(p + ".se_block.conv2.conv", C, se_channels, 1)
    tdnn("mfa", mfa_channels, n_blocks * C, 1)
    tdnn("asp.tdnn", att_channels, 3 * mfa_channels, 1)
    conv("asp.conv.conv", mfa_channels, att_channels, 1)
    bn("asp_bn.norm", 2 * mfa_channels)
    conv("fc.conv", emb_dim, 2 * mfa_channels, 1)
    m = {"arch": "ecapa_tdnn", "sd": sd, "n_mels": n_mels, "emb_dim": emb_dim,
         "channels": C, "n_blocks": n_blocks + 1, "scale": scale, "se_channels": se_channels,
         "att_channels": att_channels, "l2_normalize": True}
    if calibrate:
        import torch
        crng = np.random.default_rng(seed + 104729)
        feats = torch.from_numpy(crng.standard_normal((8, n_mels, 160)) * 1.5)
        ecapa_forward_torch(m, feats, calibrate=True)
    return m


def tiny_ecapa_model(seed: int = 0, n_mels: int = 16) -> dict:
    """Narrow ECAPA (same topology rules) for CPU tests: C 64, scale 4, 3 blocks."""
    return ecapa_model(seed, n_mels=n_mels, channels=64, scale=4, se_channels=16,
                       mfa_channels=96, att_channels=32, emb_dim=32)


def ecapa_forward_torch(m: dict, feats, calibrate: bool = False):
    """ECAPA-TDNN forward in torch float64 with SpeechBrain semantics, written with
    torch's own reflect padding, conv1d, batch_norm and softmax (an implementation
    independent of the numpy oracle). feats: [N, n_mels, T] (CMN already applied).
    Returns (embedding, pre-norm embedding), each [N, emb_dim].

    calibrate=True first sets each BatchNorm's running statistics (in execution
    order) to the mean / variance of its input over the batch and time, then
    applies it; the updated arrays are written back into m["sd"]."""
    import torch
    import torch.nn.functional as Fn

    sd = m["sd"]

    def t(name):
        return torch.from_numpy(sd[name].astype(np.float64))

    def conv(x, p, dil=1):
        wt = t(p + ".weight")
        k = wt.shape[-1]
        pad = (k - 1) // 2 * dil
        if pad:
            x = Fn.pad(x, (pad, pad), mode="reflect")
        return Fn.conv1d(x, wt, t(p + ".bias"), dilation=dil)

    def bn(x, p):
        if calibrate:
            dims = (0, 2) if x.dim() == 3 else (0,)
            mu = x.mean(dims)
            var = x.var(dims, unbiased=False).clamp_min(1e-2)
            sd[p + ".running_mean"] = mu.numpy().astype(np.float32)
            sd[p + ".running_var"] = var.numpy().astype(np.float32)
        return Fn.batch_norm(x, t(p + ".running_mean"), t(p + ".running_var"), t(p + ".weight"),
                             t(p + ".bias"), training=False, eps=1e-5)

    def tdnn(x, p, dil=1):
        return bn(torch.relu(conv(x, p + ".conv.conv", dil)), p + ".norm.norm")

    def block(x, i):
        p = f"blocks.{i}"
        res = x
        h = tdnn(x, p + ".tdnn1")
        s = int(m["scale"])
        parts = torch.chunk(h, s, dim=1)
        ys = [parts[0]]
        for j in range(1, s):
            inp = parts[j] if j == 1 else parts[j] + ys[-1]
            ys.append(tdnn(inp, f"{p}.res2net_block.blocks.{j - 1}", dil=i + 1))
        h = tdnn(torch.cat(ys, 1), p + ".tdnn2")
        g = h.mean(2, keepdim=True)
        g = torch.relu(conv(g, p + ".se_block.conv1.conv"))
        g = torch.sigmoid(conv(g, p + ".se_block.conv2.conv"))
        return h * g + res

    with torch.no_grad():
        x = tdnn(feats.to(torch.float64), "blocks.0")
        outs = []
        for i in range(1, int(m["n_blocks"])):
            x = block(x, i)
            outs.append(x)
        x = tdnn(torch.cat(outs, 1), "mfa")
        T = x.shape[2]
        mean = x.mean(2, keepdim=True)
        std = ((x - mean) ** 2).mean(2, keepdim=True).clamp_min(1e-12).sqrt()
        ctx = torch.cat([x, mean.expand(-1, -1, T), std.expand(-1, -1, T)], 1)
        a = torch.tanh(tdnn(ctx, "asp.tdnn"))
        a = torch.softmax(conv(a, "asp.conv.conv"), dim=2)
        mu = (a * x).sum(2)
        sdv = (a * (x - mu.unsqueeze(2)) ** 2).sum(2).clamp_min(1e-12).sqrt()
        pooled = bn(torch.cat([mu, sdv], 1), "asp_bn.norm")
        pre = conv(pooled.unsqueeze(2), "fc.conv").squeeze(2)
        emb = pre / pre.norm(dim=1, keepdim=True)
    return emb.numpy(), pre.numpy()


def f16_ecapa_model(m: dict) -> dict:
    """Round every ECAPA conv weight (not biases / BatchNorm) through f16."""
    sd = {k: (v.astype(np.float16).astype(np.float32) if k.endswith("conv.weight") else v)
          for k, v in m["sd"].items()}
    return dict(m, sd=sd)


_ECAPA_QUANT_EXCLUDE = ("fc.", "asp.")
_ECAPA_QUANT_EXCLUDE_IN = (".se_block.", ".tdnn1.", ".tdnn2.")


def _ecapa_quantizable(name: str, arr: np.ndarray) -> bool:
    """The reference converter's quant_plan (scripts/convert_voicedetect_to_gguf.py:
    allowlist '.conv.weight', exclusions fc / asp / se_block / tdnn1 / tdnn2,
    kernel 1, both channel counts >= 32): only the MFA weight qualifies."""
    if not name.endswith(".conv.weight") or arr.ndim != 3 or arr.shape[2] != 1:
        return False
    if name.startswith(_ECAPA_QUANT_EXCLUDE) or any(s in name for s in _ECAPA_QUANT_EXCLUDE_IN):
        return False
    return arr.shape[0] >= 32 and arr.shape[1] >= 32


def write_ecapa_gguf(path: str, m: dict, dtype: str = "f32") -> None:
    """Write an ecapa_tdnn GGUF with the reference's KV schema and verbatim tensor
    names. dtype f32 | f16 | q8_0 applies where the reference converter quantises
    (the 1x1 MFA weight, stored squeezed to 2-D [OC, IC]); every other tensor is f32."""
    import gguf
    from gguf import quants

    w = gguf.GGUFWriter(path, arch="voicedetect")
    w.add_string("voicedetect.arch", "ecapa_tdnn")
    w.add_uint32("voicedetect.embedding_dim", int(m["emb_dim"]))
    w.add_bool("voicedetect.l2_normalize", bool(m.get("l2_normalize", True)))
    w.add_uint32("voicedetect.fbank.sample_rate", 16000)
    w.add_uint32("voicedetect.fbank.n_mels", int(m["n_mels"]))
    w.add_uint32("voicedetect.fbank.n_fft", 512)
    w.add_uint32("voicedetect.fbank.win_length", 400)
    w.add_uint32("voicedetect.fbank.hop_length", 160)
    w.add_float32("voicedetect.fbank.preemph", 0.97)
    w.add_float32("voicedetect.fbank.low_freq", 20.0)
    w.add_float32("voicedetect.fbank.high_freq", 0.0)
    w.add_bool("voicedetect.fbank.use_energy", False)
    w.add_bool("voicedetect.fbank.cmn", True)
    w.add_string("voicedetect.fbank.window", "povey")
    w.add_uint32("voicedetect.ecapa.channels", int(m["channels"]))
    w.add_uint32("voicedetect.ecapa.n_blocks", int(m["n_blocks"]))
    w.add_uint32("voicedetect.ecapa.se_channels", int(m["se_channels"]))
    w.add_uint32("voicedetect.ecapa.res2net_scale", int(m["scale"]))
    w.add_uint32("voicedetect.ecapa.attention_channels", int(m["att_channels"]))
    for name, arr in m["sd"].items():
        arr = np.ascontiguousarray(arr, np.float32)
        if dtype == "f32" or not _ecapa_quantizable(name, arr):
            w.add_tensor(name, arr)
            continue
        a2 = np.ascontiguousarray(arr[:, :, 0])
        if dtype == "f16":
            w.add_tensor(name, a2.astype(np.float16))
        elif dtype == "q8_0" and a2.shape[1] % 32 == 0:
            qb = quants.quantize(a2, gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, qb, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif dtype == "q8_0":
            w.add_tensor(name, arr)
        else:
            raise ValueError(dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def quantized_ecapa_model(m: dict, dtype: str) -> dict:
    """The model a dtype GGUF carries (quantised MFA weight round-tripped)."""
    if dtype == "f32":
        return m
    import gguf
    from gguf import quants

    sd = dict(m["sd"])
    for name, arr in m["sd"].items():
        if not _ecapa_quantizable(name, arr):
            continue
        a2 = np.ascontiguousarray(arr[:, :, 0])
        if dtype == "f16":
            r = a2.astype(np.float16).astype(np.float32)
        elif a2.shape[1] % 32 == 0:
            qt = gguf.GGMLQuantizationType.Q8_0
            r = quants.dequantize(quants.quantize(a2, qt), qt).reshape(a2.shape)
        else:
            r = a2
        sd[name] = r[:, :, None].astype(np.float32)
    return dict(m, sd=sd)


# ---------------------------------------------------------------------------
# CAM++ (3D-Speaker D-TDNN with context-aware masking)
# ---------------------------------------------------------------------------
CAMPP_LAYERS = (12, 24, 16)
CAMPP_DIL = (1, 2, 2)


def campplus_model(seed: int = 0, n_mels: int = N_MELS, m_channels: int = 32,
                   init_channels: int = 128, growth: int = 32, bn_size: int = 4,
                   layers=CAMPP_LAYERS, emb_dim: int = 192, calibrate: bool = True) -> dict:
    """Synthetic 3D-Speaker CAM++ as the reference's manifest sees it
    (src/model_loader.hpp:82-98, src/encoder_campplus.cpp:148-300): a flat list of
    convs in forward-EXECUTION order and a list of the runtime (affine) BatchNorms:

      FCM (12 convs, BatchNorm folded, freq-axis strides): stem 3x3 1->M; two stages
        of [BasicResBlock s2 (conv1, conv2, 1x1 shortcut), BasicResBlock s1 (conv1,
        conv2)]; conv2 3x3 s2. Freq 80 -> 10, channels M x 10.
      TDNN: Conv1d k=5 stride 2 pad 2 (BN folded) -> ReLU.
      3 CAMDenseTDNN blocks (layers 12 / 24 / 16, dilation 1 / 2 / 2), each layer:
        BN (runtime) -> ReLU -> 1x1 conv to bn_size*growth (BN folded) -> ReLU -> CAM:
        linear_local k=3 dilated (no bias), linear1 1x1 (bias) -> ReLU, linear2 1x1
        (bias) -> sigmoid, on the mean + 100-frame segment context; the layer output
        (growth channels) is concatenated to the block input.
      Transits: BN (runtime) -> ReLU -> 1x1 conv halving the channels (no bias; the
        last one has the output BN folded in, a bias, and a ReLU after it).
      Head: stats pooling (mean, unbiased std), 1x1 dense 2C -> emb (no bias),
        affine-free BN.

    Weights are Kaiming-normal; with calibrate=True every BatchNorm (folded or
    runtime) takes the statistics of its input on a seeded calibration batch, as a
    trained model's running statistics are (see ecapa_model)."""
    rng = np.random.default_rng(seed)
    convs: list[dict] = []
    bns: list[dict] = []

    def conv(oc, ic, k, two_d=False, bias=True, **meta):
        shape = (oc, ic, k, k) if two_d else (oc, ic, k)
        w = (rng.standard_normal(shape) * np.sqrt(2.0 / (ic * k * (k if two_d else 1)))).astype(np.float32)
        b = rng.normal(0.0, 0.05, oc).astype(np.float32) if bias else None
        convs.append(dict(w=w, b=b, fold=bias and meta.pop("fold", True), **meta))

    def bn(c):
        bns.append({"weight": rng.uniform(0.8, 1.2, c).astype(np.float32),
                    "bias": rng.normal(0.0, 0.1, c).astype(np.float32),
                    "running_mean": rng.normal(0.0, 0.1, c).astype(np.float32),
                    "running_var": rng.uniform(0.5, 1.5, c).astype(np.float32)})

    M = m_channels
    conv(M, 1, 3, True)                                     # FCM stem
    for _ in range(2):                                      # layer1, layer2
        conv(M, M, 3, True), conv(M, M, 3, True), conv(M, M, 1, True)   # s2 block + shortcut
        conv(M, M, 3, True), conv(M, M, 3, True)                         # s1 block
    conv(M, M, 3, True)                                     # FCM conv2 (s2)
    f = n_mels
    for _ in range(3):
        f = (f - 1) // 2 + 1
    conv(init_channels, M * f, 5)                           # TDNN
    C = init_channels
    bnc = bn_size * growth
    for bi, nl in enumerate(layers):
        for _ in range(nl):
            bn(C)                                           # nonlinear1
            conv(bnc, C, 1)                                 # linear1 (+ folded BN)
            conv(growth, bnc, 3, bias=False)                # CAM linear_local
            conv(bnc // 2, bnc, 1, fold=False)              # CAM linear1 (genuine bias)
            conv(growth, bnc // 2, 1, fold=False)           # CAM linear2 (genuine bias)
            C += growth
        bn(C)                                               # transit nonlinear
        conv(C // 2, C, 1, bias=(bi == 2))                  # transit (last: + out BN)
        C //= 2
    conv(emb_dim, 2 * C, 1, bias=False)                     # dense head
    m = {"arch": "campplus", "convs": convs, "bns": bns, "n_mels": n_mels, "emb_dim": emb_dim,
         "emb_bn_mean": rng.normal(0.0, 0.1, emb_dim).astype(np.float32),
         "emb_bn_var": rng.uniform(0.5, 1.5, emb_dim).astype(np.float32),
         "bn_eps": 1e-5, "l2_normalize": True, "layers": list(layers)}
    assert len(convs) == 12 + 1 + 4 * sum(layers) + 3 + 1
    if calibrate:
        import torch
        crng = np.random.default_rng(seed + 15485863)
        feats = torch.from_numpy(crng.standard_normal((6, n_mels, 240)) * 1.5)
        campplus_forward_torch(m, feats, calibrate=True)
    return m


def tiny_campplus_model(seed: int = 0, n_mels: int = 80) -> dict:
    """Narrow CAM++ for CPU tests: same topology rules, 2 / 3 / 2 dense layers."""
    return campplus_model(seed, n_mels=n_mels, m_channels=16, init_channels=64, growth=16,
                          bn_size=2, layers=(2, 3, 2), emb_dim=48)


def campplus_forward_torch(m: dict, feats, calibrate: bool = False):
    """CAM++ forward in torch float64 with the reference's semantics, written with
    torch's own conv1d / conv2d / batch_norm (an implementation independent of the
    numpy oracle). feats [N, n_mels, T] (CMN applied). Returns (emb, pre-norm) [N, D].
    calibrate=True folds measured BatchNorm statistics into the BN-folded convs and
    sets the runtime BatchNorms' running statistics, in execution order."""
    import torch
    import torch.nn.functional as Fn

    convs, bns = m["convs"], m["bns"]
    ci = [0]
    bi = [0]
    eps = float(m["bn_eps"])

    def t(a):
        return torch.from_numpy(np.asarray(a, np.float64))

    def fold(c, y, dims):
        # calibrated BatchNorm folded into a biased conv: w *= s, b = beta - mu * s
        mu = y.mean(dims)
        s = 1.0 / torch.sqrt(y.var(dims, unbiased=False) + 1e-5)
        beta = t(np.random.default_rng(len(c["w"].ravel())).normal(0.0, 0.1, y.shape[1]))
        shp = (-1,) + (1,) * (c["w"].ndim - 1)
        c["w"] = (t(c["w"]) * s.view(shp)).numpy().astype(np.float32)
        c["b"] = (beta - mu * s).numpy().astype(np.float32)

    def conv2d(x, stride_f):
        c = convs[ci[0]]
        ci[0] += 1
        k = c["w"].shape[-1]
        pad = (k - 1) // 2
        if calibrate and c["b"] is not None and c["fold"]:
            y = Fn.conv2d(x, t(c["w"]), None, stride=(stride_f, 1), padding=pad)
            fold(c, y, (0, 2, 3))
        return Fn.conv2d(x, t(c["w"]), None if c["b"] is None else t(c["b"]),
                         stride=(stride_f, 1), padding=pad)

    def conv1d(x, stride=1, pad=0, dil=1):
        c = convs[ci[0]]
        ci[0] += 1
        if calibrate and c["b"] is not None and c["fold"]:
            y = Fn.conv1d(x, t(c["w"]), None, stride=stride, padding=pad, dilation=dil)
            fold(c, y, (0, 2))
        return Fn.conv1d(x, t(c["w"]), None if c["b"] is None else t(c["b"]),
                         stride=stride, padding=pad, dilation=dil)

    def bn(x):
        p = bns[bi[0]]
        bi[0] += 1
        if calibrate:
            p["running_mean"] = x.mean((0, 2)).numpy().astype(np.float32)
            p["running_var"] = x.var((0, 2), unbiased=False).clamp_min(1e-2).numpy().astype(np.float32)
        return Fn.batch_norm(x, t(p["running_mean"]), t(p["running_var"]), t(p["weight"]),
                             t(p["bias"]), training=False, eps=eps)

    def block(x, stride):
        out = torch.relu(conv2d(x, stride))
        out = conv2d(out, 1)
        sc = conv2d(x, stride) if stride != 1 else x
        return torch.relu(out + sc)

    with torch.no_grad():
        x = feats.to(torch.float64).unsqueeze(1)            # [N, 1, F, T]
        h = torch.relu(conv2d(x, 1))
        h = block(h, 2)
        h = block(h, 1)
        h = block(h, 2)
        h = block(h, 1)
        h = torch.relu(conv2d(h, 2))
        N, Cc, Fq, T = h.shape
        h = h.reshape(N, Cc * Fq, T)                         # channel = c * F' + f
        h = torch.relu(conv1d(h, stride=2, pad=2))
        Tp = h.shape[-1]
        seg = torch.arange(Tp) // 100
        nseg = (Tp + 99) // 100
        for blk, (nl, dil) in enumerate(zip(m["layers"], CAMPP_DIL)):
            for _ in range(nl):
                a = torch.relu(bn(h))
                cc = torch.relu(conv1d(a))
                y = conv1d(cc, pad=dil, dil=dil)
                # context: global mean + 100-frame segment means (each divided by 100)
                segs = torch.stack([cc[:, :, s * 100:(s + 1) * 100].sum(-1) / 100.0
                                    for s in range(nseg)], -1)           # [N, C, nseg]
                ctx = cc.mean(-1, keepdim=True) + segs[:, :, seg]
                mk = torch.sigmoid(conv1d(torch.relu(conv1d(ctx))))
                h = torch.cat([h, y * mk], 1)
            tr = conv1d(torch.relu(bn(h)))
            h = torch.relu(tr) if blk == 2 else tr
        mean = h.mean(-1)
        std = h.std(-1, unbiased=True) if Tp > 1 else torch.zeros_like(mean)
        stats = torch.cat([mean, std], 1).unsqueeze(-1)
        e = conv1d(stats).squeeze(-1)
        if calibrate:
            m["emb_bn_mean"] = e.mean(0).numpy().astype(np.float32)
            m["emb_bn_var"] = e.var(0, unbiased=False).clamp_min(1e-2).numpy().astype(np.float32)
        pre = (e - t(m["emb_bn_mean"])) / torch.sqrt(t(m["emb_bn_var"]) + eps)
        emb = pre / pre.norm(dim=1, keepdim=True)
    assert ci[0] == len(convs) and bi[0] == len(bns)
    return emb.numpy(), pre.numpy()


def write_campplus_gguf(path: str, m: dict, dtype: str = "f32") -> None:
    """campplus GGUF with the reference's manifest keys (voicedetect.campplus.*,
    src/model_loader.cpp:165-172). dtype f32 | f16 (conv weights) | q8_0 (the 1x1
    Conv1d weights whose input width is a multiple of 32 squeezed to [OC, IC] and
    quantised, the converter's rule for rank <= 3 weights; the other convs f16)."""
    import gguf
    from gguf import quants

    w = gguf.GGUFWriter(path, arch="voicedetect")
    w.add_string("voicedetect.arch", "campplus")
    w.add_uint32("voicedetect.embedding_dim", int(m["emb_dim"]))
    w.add_bool("voicedetect.l2_normalize", bool(m.get("l2_normalize", True)))
    w.add_uint32("voicedetect.fbank.sample_rate", 16000)
    w.add_uint32("voicedetect.fbank.n_mels", int(m["n_mels"]))
    w.add_uint32("voicedetect.fbank.n_fft", 512)
    w.add_uint32("voicedetect.fbank.win_length", 400)
    w.add_uint32("voicedetect.fbank.hop_length", 160)
    w.add_float32("voicedetect.fbank.preemph", 0.97)
    w.add_float32("voicedetect.fbank.low_freq", 20.0)
    w.add_float32("voicedetect.fbank.high_freq", 0.0)
    w.add_bool("voicedetect.fbank.cmn", True)
    wn, bn_ = [], []
    tensors = []
    for i, c in enumerate(m["convs"]):
        wn.append(f"conv{i}.weight")
        tensors.append((wn[-1], c["w"], "conv"))
        if c["b"] is not None:
            bn_.append(f"conv{i}.bias")
            tensors.append((bn_[-1], c["b"], "bias"))
        else:
            bn_.append("")
    pre = []
    for j, b in enumerate(m["bns"]):
        pre.append(f"bn{j}")
        for k in ("weight", "bias", "running_mean", "running_var"):
            tensors.append((f"bn{j}.{k}", b[k], "bias"))
    tensors.append(("emb_bn.running_mean", m["emb_bn_mean"], "bias"))
    tensors.append(("emb_bn.running_var", m["emb_bn_var"], "bias"))
    w.add_array("voicedetect.campplus.conv_weight", wn)
    w.add_array("voicedetect.campplus.conv_bias", bn_)
    w.add_array("voicedetect.campplus.bn_prefix", pre)
    w.add_string("voicedetect.campplus.emb_bn_mean", "emb_bn.running_mean")
    w.add_string("voicedetect.campplus.emb_bn_var", "emb_bn.running_var")
    w.add_float32("voicedetect.campplus.bn_eps", float(m["bn_eps"]))
    for name, arr, kind in tensors:
        arr = np.ascontiguousarray(arr, np.float32)
        if dtype == "q8_0" and kind == "conv" and _campplus_q8(arr):
            qb = quants.quantize(np.ascontiguousarray(arr[:, :, 0]), gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, qb, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif dtype in ("f16", "q8_0") and kind == "conv" and arr.shape[1] > 1:
            w.add_tensor(name, arr.astype(np.float16))
        else:
            w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def f16_campplus_model(m: dict) -> dict:
    """The weights an f16 GGUF carries (conv weights with IC > 1 rounded)."""
    convs = [dict(c, w=c["w"].astype(np.float16).astype(np.float32)) if c["w"].shape[1] > 1
             else c for c in m["convs"]]
    return dict(m, convs=convs)


def _campplus_q8(w: np.ndarray) -> bool:
    """A 1x1 Conv1d weight [OC, IC, 1] whose rows split into q8_0 blocks of 32."""
    return w.ndim == 3 and w.shape[2] == 1 and w.shape[1] % 32 == 0


def q8_campplus_model(m: dict) -> dict:
    """The weights a q8_0 GGUF carries: quantisable 1x1 convs round-tripped through
    q8_0, the other convs with IC > 1 through f16."""
    import gguf
    from gguf import quants
    qt = gguf.GGMLQuantizationType.Q8_0
    convs = []
    for c in m["convs"]:
        w = c["w"]
        if _campplus_q8(w):
            a2 = np.ascontiguousarray(w[:, :, 0], np.float32)
            r = quants.dequantize(quants.quantize(a2, qt), qt).reshape(a2.shape)
            convs.append(dict(c, w=r[:, :, None].astype(np.float32)))
        elif w.shape[1] > 1:
            convs.append(dict(c, w=w.astype(np.float16).astype(np.float32)))
        else:
            convs.append(c)
    return dict(m, convs=convs)
