"""ECAPA-TDNN CPU oracle (TEST INFRASTRUCTURE: only tests/, smoke() and bench.py's
CPU legs use it; the product path never does).

A numpy float32 restatement of the reference's EcapaEncoder, op for op
(src/encoder.cpp). The reference builds it from ggml graph ops (im2col +
mul_mat, get_rows for the reflect padding, mean, soft_max, ...) that live in the
absent ggml submodule, and its tests need real SpeechBrain weights that are not
shipped, so this restatement cannot be pinned to the reference itself. It is
pinned instead against a second, independent formulation: torch's reflect pad,
conv1d, batch_norm and softmax in float64 (vd_synth.ecapa_forward_torch), through
the golden vectors tests/golden/ref_ecapa_tiny.npz.

Arithmetic follows the reference: float32 tensors and matmuls (ggml's f32 path),
BatchNorm folded to scale / shift in float32, L2 normalisation in float64 on the
host.
"""
from __future__ import annotations

import numpy as np

BN_EPS = np.float32(1e-5)    # src/encoder.cpp:13
ASP_EPS = np.float32(1e-12)  # src/encoder.cpp:19


def reflect_index(T: int, pad: int) -> np.ndarray:
    """Time index list of reflect_pad_time (src/encoder.cpp:32-50)."""
    idx = np.empty(T + 2 * pad, np.int64)
    for j in range(T + 2 * pad):
        if j < pad:
            t = pad - j
        elif j < pad + T:
            t = j - pad
        else:
            t = (T - 2) - (j - pad - T)
        idx[j] = t
    if T + 2 * pad and (idx.min() < 0 or idx.max() >= T):
        raise ValueError(f"reflect padding by {pad} needs more than {pad} frames (T={T})")
    return idx


def conv1d_same(w: np.ndarray, b: np.ndarray | None, x: np.ndarray, dil: int = 1) -> np.ndarray:
    """Conv1d with "same" reflect padding, stride 1 (src/encoder.cpp:65-110).
    w: [OC, IC, K] f32 (torch order), x: [IC, T] -> [OC, T]."""
    oc, ic, k = w.shape
    T = x.shape[1]
    if k == 1:
        y = w[:, :, 0] @ x
    else:
        pad = (k - 1) // 2 * dil
        xp = x[:, reflect_index(T, pad)]
        cols = np.concatenate([xp[:, j * dil:j * dil + T] for j in range(k)], axis=0)
        y = np.ascontiguousarray(w.transpose(0, 2, 1)).reshape(oc, k * ic) @ cols
    if b is not None:
        y = y + b[:, None]
    return y.astype(np.float32)


def bn1d_eval(sd: dict, p: str, x: np.ndarray) -> np.ndarray:
    """Eval BatchNorm folded to scale / shift in f32 (src/encoder.cpp:125-151)."""
    g, beta = sd[p + ".weight"], sd[p + ".bias"]
    mu, var = sd[p + ".running_mean"], sd[p + ".running_var"]
    scale = (g / np.sqrt(var + BN_EPS)).astype(np.float32)
    shift = (beta - scale * mu).astype(np.float32)
    if x.ndim == 1:
        return (x * scale + shift).astype(np.float32)
    return (x * scale[:, None] + shift[:, None]).astype(np.float32)


def tdnn_block(sd: dict, p: str, x: np.ndarray, dil: int = 1) -> np.ndarray:
    """Conv1d -> ReLU -> BatchNorm1d (src/encoder.cpp:157-167)."""
    h = conv1d_same(sd[p + ".conv.conv.weight"], sd[p + ".conv.conv.bias"], x, dil)
    return bn1d_eval(sd, p + ".norm.norm", np.maximum(h, 0.0))


def res2net_block(sd: dict, p: str, x: np.ndarray, scale: int, dil: int) -> np.ndarray:
    """Hierarchical residual groups (src/encoder.cpp:174-194)."""
    g = x.shape[0] // scale
    out, prev = [], None
    for i in range(scale):
        xi = x[i * g:(i + 1) * g]
        if i == 0:
            yi = xi
        else:
            inp = xi if i == 1 else (xi + prev).astype(np.float32)
            yi = tdnn_block(sd, f"{p}.blocks.{i - 1}", inp, dil)
        out.append(yi)
        prev = yi
    return np.concatenate(out, axis=0)


def se_block(sd: dict, p: str, x: np.ndarray) -> np.ndarray:
    """Squeeze-excitation (src/encoder.cpp:196-209)."""
    s = x.mean(axis=1, keepdims=True, dtype=np.float32)
    s = conv1d_same(sd[p + ".conv1.conv.weight"], sd[p + ".conv1.conv.bias"], s)
    s = np.maximum(s, 0.0)
    s = conv1d_same(sd[p + ".conv2.conv.weight"], sd[p + ".conv2.conv.bias"], s)
    s = (1.0 / (1.0 + np.exp(-s))).astype(np.float32)
    return (x * s).astype(np.float32)


def se_res2net_block(sd: dict, idx: int, x: np.ndarray, dil: int) -> np.ndarray:
    """tdnn1 -> res2net -> tdnn2 -> SE -> + input (src/encoder.cpp:211-230)."""
    p = f"blocks.{idx}"
    h = tdnn_block(sd, p + ".tdnn1", x)
    scale = 1
    while f"{p}.res2net_block.blocks.{scale - 1}.conv.conv.weight" in sd:
        scale += 1
    h = res2net_block(sd, p + ".res2net_block", h, scale, dil)
    h = tdnn_block(sd, p + ".tdnn2", h)
    h = se_block(sd, p + ".se_block", h)
    return (h + x).astype(np.float32)


def attentive_stat_pooling(sd: dict, x: np.ndarray) -> np.ndarray:
    """Global-context ASP (src/encoder.cpp:246-286): returns [2C] = (mu, sd)."""
    T = x.shape[1]
    gmean = x.mean(axis=1, keepdims=True, dtype=np.float32)
    gvar = ((x - gmean) ** 2).mean(axis=1, keepdims=True, dtype=np.float32)
    gstd = np.sqrt(np.clip(gvar, ASP_EPS, np.float32(1e30)))
    ctx = np.concatenate([x, np.repeat(gmean, T, 1), np.repeat(gstd, T, 1)], axis=0)
    a = np.tanh(tdnn_block(sd, "asp.tdnn", ctx))
    a = conv1d_same(sd["asp.conv.conv.weight"], sd["asp.conv.conv.bias"], a)
    a = np.exp(a - a.max(axis=1, keepdims=True))
    a = (a / a.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    mu = (a * x).sum(axis=1, dtype=np.float32)
    var = (a * (x - mu[:, None]) ** 2).sum(axis=1, dtype=np.float32)
    sdv = np.sqrt(np.clip(var, ASP_EPS, np.float32(1e30)))
    return np.concatenate([mu, sdv]).astype(np.float32)


def ecapa_embed(m: dict, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """EcapaEncoder::run_forward (src/encoder.cpp:288-373). feats: [n_mels, T]
    (FBank with CMN). Returns (embedding, pre-norm embedding)."""
    sd = m["sd"]
    x = np.ascontiguousarray(feats, np.float32)
    h = tdnn_block(sd, "blocks.0", x)
    outs = []
    i = 1
    while f"blocks.{i}.tdnn1.conv.conv.weight" in sd:
        h = se_res2net_block(sd, i, h, i + 1)
        outs.append(h)
        i += 1
    h = tdnn_block(sd, "mfa", np.concatenate(outs, axis=0))
    pooled = attentive_stat_pooling(sd, h)
    normed = bn1d_eval(sd, "asp_bn.norm", pooled)
    pre = conv1d_same(sd["fc.conv.weight"], sd["fc.conv.bias"], normed[:, None])[:, 0]
    pre = pre.astype(np.float32)
    emb = pre
    if m.get("l2_normalize", True):
        n = np.sqrt(np.sum(pre.astype(np.float64) ** 2))
        if n > 0:
            emb = (pre.astype(np.float64) / n).astype(np.float32)
    return emb, pre
