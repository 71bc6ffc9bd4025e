"""CAM++ CPU oracle (TEST INFRASTRUCTURE: only tests/, smoke() and bench.py's CPU legs
use it; the product path never does).

A numpy float32 restatement of the reference's CamPPlusEncoder, op for op
(src/encoder_campplus.cpp:148-300). Like the ECAPA oracle it cannot be pinned to
the reference itself (the graph runs on the absent ggml library and the reference's
CAM++ test needs ONNX weights that are not shipped); it is pinned to an independent
float64 torch formulation (vd_synth.campplus_forward_torch) through the golden
vectors tests/golden/ref_campplus_tiny.npz.
"""
from __future__ import annotations

import numpy as np

from .ecapa import BN_EPS  # noqa: F401  (same PyTorch default)

SEG = 100               # CAM context segment length (src/encoder_campplus.cpp:162-181)
DIL = (1, 2, 2)         # dilation per CAMDenseTDNN block (:184-185)


def conv2d_freq(x: np.ndarray, w: np.ndarray, b: np.ndarray | None, stride_f: int) -> np.ndarray:
    """FCM Conv2d (next_conv2d, :57-65): x [IC, F, T], w [OC, IC, K, K] (freq, time),
    stride on the frequency axis only, zero padding (K-1)/2."""
    oc, ic, k, _ = w.shape
    pad = (k - 1) // 2
    _, F, T = x.shape
    xp = np.pad(x, ((0, 0), (pad, pad), (pad, pad)))
    Fo = (F + 2 * pad - k) // stride_f + 1
    cols = np.empty((ic, k, k, Fo, T), np.float32)
    for kf in range(k):
        for kt in range(k):
            cols[:, kf, kt] = xp[:, kf:kf + stride_f * (Fo - 1) + 1:stride_f, kt:kt + T]
    y = w.reshape(oc, ic * k * k) @ cols.reshape(ic * k * k, Fo * T)
    y = y.reshape(oc, Fo, T)
    if b is not None:
        y = y + b[:, None, None]
    return y.astype(np.float32)


def conv1d(x: np.ndarray, w: np.ndarray, b: np.ndarray | None, stride: int = 1, pad: int = 0,
           dil: int = 1) -> np.ndarray:
    """next_conv1d (:27-50): x [IC, T] channel-major, w [OC, IC, K], zero padding."""
    oc, ic, k = w.shape
    T = x.shape[1]
    if k == 1 and stride == 1 and pad == 0:
        y = w[:, :, 0] @ x
    else:
        xp = np.pad(x, ((0, 0), (pad, pad)))
        To = (T + 2 * pad - dil * (k - 1) - 1) // stride + 1
        cols = np.stack([xp[:, j * dil:j * dil + stride * (To - 1) + 1:stride] for j in range(k)], 1)
        y = w.reshape(oc, ic * k) @ cols.reshape(ic * k, To)
    if b is not None:
        y = y + b[:, None]
    return y.astype(np.float32)


def bn_affine(p: dict, eps: float) -> tuple[np.ndarray, np.ndarray]:
    """bn1d / bn1d_cm (:72-133): eval BatchNorm as f32 scale / shift."""
    scale = (p["weight"] / np.sqrt(p["running_var"] + np.float32(eps))).astype(np.float32)
    shift = (p["bias"] - scale * p["running_mean"]).astype(np.float32)
    return scale, shift


def campplus_embed(m: dict, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """CamPPlusEncoder::forward_capture (:148-300). feats [n_mels, T] (FBank with CMN).
    Returns (embedding, pre-norm embedding)."""
    convs, bns = m["convs"], m["bns"]
    eps = float(m["bn_eps"])
    ci = iter(range(len(convs)))
    bi = iter(range(len(bns)))

    def cv():
        c = convs[next(ci)]
        return c["w"], c["b"]

    relu = lambda a: np.maximum(a, np.float32(0.0))  # noqa: E731

    # FCM (:203-230): stem, 2 x (s2 block, s1 block), conv2 s2
    x = np.ascontiguousarray(feats, np.float32)[None]          # [1, F, T]
    h = relu(conv2d_freq(x, *cv(), 1))

    def block(x, stride):
        out = relu(conv2d_freq(x, *cv(), stride))
        out = conv2d_freq(out, *cv(), 1)
        sc = conv2d_freq(x, *cv(), stride) if stride != 1 else x
        return relu(out + sc)

    for s in (2, 1, 2, 1):
        h = block(h, s)
    h = relu(conv2d_freq(h, *cv(), 2))
    C, Fq, T = h.shape
    h = h.reshape(C * Fq, T)                                     # channel = c * F' + f (:232-236)
    h = relu(conv1d(h, *cv(), stride=2, pad=2))                  # TDNN (:238-241)
    Tp = h.shape[1]
    nseg = (Tp + SEG - 1) // SEG
    seg = np.arange(Tp) // SEG
    for blk, nl in enumerate(m["layers"]):
        dil = DIL[blk]
        for _ in range(nl):
            sc, sh = bn_affine(bns[next(bi)], eps)
            a = relu(h * sc[:, None] + sh[:, None])
            cc = relu(conv1d(a, *cv()))
            y = conv1d(cc, *cv(), pad=dil, dil=dil)
            # context = global mean + 100-frame segment sums / 100 (:162-181, :266-270)
            g = cc.sum(1, dtype=np.float32) / np.float32(Tp)
            segm = np.stack([cc[:, s * SEG:(s + 1) * SEG].sum(1, dtype=np.float32) / np.float32(SEG)
                             for s in range(nseg)], 1)
            ctx = (g[:, None] + segm[:, seg]).astype(np.float32)
            mk = relu(conv1d(ctx, *cv()))
            mk = conv1d(mk, *cv())
            mk = (1.0 / (1.0 + np.exp(-mk))).astype(np.float32)
            h = np.concatenate([h, (y * mk).astype(np.float32)], 0)
        sc, sh = bn_affine(bns[next(bi)], eps)
        t = conv1d(relu(h * sc[:, None] + sh[:, None]), *cv())
        h = relu(t) if blk == 2 else t
    # stats pooling: mean + unbiased std, no eps (:283-292)
    mean = h.mean(1, dtype=np.float32)
    var = ((h - mean[:, None]) ** 2).mean(1, dtype=np.float32)
    if Tp > 1:
        var = (var * np.float32(Tp / (Tp - 1))).astype(np.float32)
    stats = np.concatenate([mean, np.sqrt(var)]).astype(np.float32)
    w, _ = cv()
    e = (w[:, :, 0] @ stats).astype(np.float32)                 # dense, no bias (:294-298)
    s = (1.0 / np.sqrt(m["emb_bn_var"] + np.float32(eps))).astype(np.float32)
    pre = (e * s - s * m["emb_bn_mean"]).astype(np.float32)     # affine-free BN (:301-302)
    emb = pre
    if m.get("l2_normalize", True):
        n = np.sqrt(np.sum(pre.astype(np.float64) ** 2))
        if n > 0:
            emb = (pre.astype(np.float64) / n).astype(np.float32)
    return emb, pre
