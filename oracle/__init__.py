"""CPU oracle for the voice-detect conv + FBank hot path (TEST INFRASTRUCTURE).

This package is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.

Two native libraries are wrapped here, both built by ``oracle/Makefile``:

* ``_build/libvdoracle.so`` -- ``vd_oracle.c``, a plain-C restatement of the
  reference algorithms (FBank ``src/fbank.cpp:121-205``, direct conv
  ``src/directconv.cpp``, ResNet34 ``src/encoder_resnet.cpp:94-185``);
* ``_ref/libvdref.so`` -- the reference's own ``src/directconv.cpp``,
  ``src/winograd.cpp`` and ``src/fbank.cpp`` compiled unmodified against a
  ggml shim, plus a restated ResNet34 graph glue around them.

Parity status: the FBank and every conv op are pinned against the reference's
own compiled kernels (tests/test_oracle.py) and FBank against torchaudio golden
vectors (tests/golden/). The pooling/FC tail uses ggml ops from the absent ggml
submodule, so it is restated (f32 with f64 accumulation) and parity is
unpinned at that boundary.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libvdoracle.so"
REF_SO = HERE / "_ref" / "libvdref.so"

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int)


def _fp(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


class ResNetDesc(C.Structure):
    _fields_ = [
        ("n_blocks", C.c_int),
        ("stem_w", _f32p), ("stem_b", _f32p), ("stem_oc", C.c_int),
        ("conv1_w", C.POINTER(_f32p)), ("conv1_b", C.POINTER(_f32p)),
        ("conv2_w", C.POINTER(_f32p)), ("conv2_b", C.POINTER(_f32p)),
        ("down_w", C.POINTER(_f32p)), ("down_b", C.POINTER(_f32p)),
        ("in_ch", _i32p), ("out_ch", _i32p), ("stride", _i32p),
        ("seg_w", _f32p), ("seg_b", _f32p), ("mean_vec", _f32p),
        ("emb_dim", C.c_int), ("pooled_dim", C.c_int),
        ("var_eps", C.c_float), ("l2_normalize", C.c_int),
    ]


def build(quiet: bool = True) -> None:
    """Compile the oracle libraries (``make -C oracle``). The reference-source
    library is only (re)built where the reference checkout exists."""
    import subprocess
    out = subprocess.run(["make", "-C", str(HERE), "-j8"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _load(path: Path) -> C.CDLL:
    if not path.exists():
        build()
    return C.CDLL(str(path))


_lib_oracle: C.CDLL | None = None
_lib_ref: C.CDLL | None = None


def lib() -> C.CDLL:
    global _lib_oracle
    if _lib_oracle is None:
        L = _load(ORACLE_SO)
        L.vdo_fbank.restype = C.c_int
        L.vdo_fbank.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_float, C.c_float, C.c_float, C.c_int, _f32p, C.c_long,
                                _i32p]
        L.vdo_conv2d.restype = None
        L.vdo_conv2d.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int, C.c_int,
                                 C.c_int, C.c_int, _f32p, C.c_int, _f32p]
        L.vdo_resnet34_forward.restype = C.c_int
        L.vdo_resnet34_forward.argtypes = [C.POINTER(ResNetDesc), _f32p, C.c_int, C.c_int,
                                           _f32p, _f32p]
        L.vdo_resample_linear.restype = C.c_long
        L.vdo_resample_linear.argtypes = [_f32p, C.c_long, C.c_int, C.c_int, _f32p, C.c_long]
        L.vdo_identify.restype = None
        L.vdo_identify.argtypes = [_f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, _i32p,
                                   _f32p]
        _lib_oracle = L
    return _lib_oracle


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> C.CDLL:
    global _lib_ref
    if _lib_ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} missing: build it with `make -C oracle ref` "
                                    "where the reference checkout is present")
        L = C.CDLL(str(REF_SO))
        L.vdref_set_threads.argtypes = [C.c_int]
        L.vdref_get_threads.restype = C.c_int
        L.vdref_fbank.restype = C.c_int
        L.vdref_fbank.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_float, C.c_float, C.c_float, C.c_int, _f32p, C.c_long,
                                  _i32p]
        for nm in ("vdref_conv3x3_blocked", "vdref_conv1x1_blocked"):
            f = getattr(L, nm)
            f.restype = None
            f.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int, _f32p, C.c_int,
                          C.c_int, _f32p]
        for nm in ("vdref_directconv3x3", "vdref_winograd3x3"):
            f = getattr(L, nm)
            f.restype = None
            f.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int, _f32p]
        L.vdref_resnet34_new.restype = C.c_void_p
        L.vdref_resnet34_new.argtypes = [C.POINTER(ResNetDesc)]
        L.vdref_resnet34_forward.restype = C.c_int
        L.vdref_resnet34_forward.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int, _f32p, _f32p]
        L.vdref_resample_linear.restype = C.c_long
        L.vdref_resample_linear.argtypes = [_f32p, C.c_long, C.c_int, C.c_int, _f32p, C.c_long]
        L.vdref_load_audio_16k_mono.restype = C.c_long
        L.vdref_load_audio_16k_mono.argtypes = [C.c_char_p, _f32p, C.c_long]
        L.vdref_drwav_decode_f32.restype = C.c_long
        L.vdref_drwav_decode_f32.argtypes = [C.c_char_p, _f32p, C.c_long, _i32p, _i32p]
        n = int(os.environ.get("VD_ORACLE_THREADS", "0")) or (os.cpu_count() or 1)
        L.vdref_set_threads(n)
        _lib_ref = L
    return _lib_ref


# ---------------------------------------------------------------------------
# FBank
# ---------------------------------------------------------------------------
FBANK_DEFAULTS = dict(sample_rate=16000, n_mels=80, n_fft=512, win=400, hop=160,
                      preemph=0.97, low_freq=20.0, high_freq=0.0, cmn=True)


def n_frames(n_samples: int, win: int = 400, hop: int = 160) -> int:
    return 0 if n_samples < win else 1 + (n_samples - win) // hop


def _fbank_call(fn, pcm: np.ndarray, **kw) -> np.ndarray:
    p = dict(FBANK_DEFAULTS, **kw)
    pcm = np.ascontiguousarray(pcm, dtype=np.float32)
    T = n_frames(len(pcm), p["win"], p["hop"])
    out = np.zeros((p["n_mels"], max(T, 1)), dtype=np.float32)
    t_out = C.c_int(0)
    rc = fn(_fp(pcm), len(pcm), p["sample_rate"], p["n_mels"], p["n_fft"], p["win"], p["hop"],
            p["preemph"], p["low_freq"], p["high_freq"], int(p["cmn"]), _fp(out), out.size,
            C.byref(t_out))
    if rc == 1:
        return np.zeros((p["n_mels"], 0), dtype=np.float32)
    if rc != 0:
        raise RuntimeError(f"fbank rc={rc}")
    assert t_out.value == T
    return out[:, :T]


def fbank(pcm: np.ndarray, **kw) -> np.ndarray:
    """C restatement of FBank::compute -> feat-major [n_mels, T] (post-CMN)."""
    return _fbank_call(lib().vdo_fbank, pcm, **kw)


def ref_fbank(pcm: np.ndarray, **kw) -> np.ndarray:
    """The reference's own FBank::compute (src/fbank.cpp) -> [n_mels, T]."""
    return _fbank_call(ref_lib().vdref_fbank, pcm, **kw)


# ---------------------------------------------------------------------------
# Convolutions (activations NCHW in numpy order (C, H, W); ggml [W, H, C])
# ---------------------------------------------------------------------------
def _out_hw(H: int, W: int, k: int, stride: int, pad: int) -> tuple[int, int]:
    return (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1


def conv2d(x: np.ndarray, w: np.ndarray, stride: int = 1, bias: np.ndarray | None = None,
           relu: bool = False) -> np.ndarray:
    """C restatement of the direct conv. x (IC, H, W) f32, w torch (OC, IC, k, k)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    IC, H, W = x.shape
    OC, _, k, _ = w.shape
    pad = (k - 1) // 2
    Ho, Wo = _out_hw(H, W, k, stride, pad)
    y = np.zeros((OC, Ho, Wo), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().vdo_conv2d(_fp(x), W, H, IC, _fp(w), OC, k, stride, pad, _fp(b), int(relu), _fp(y))
    return y


def ref_conv3x3(x: np.ndarray, w: np.ndarray, stride: int = 1, bias: np.ndarray | None = None,
                relu: bool = False) -> np.ndarray:
    """Reference blocked_conv3x3 (src/directconv.cpp:1496-1508), pad 1."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    IC, H, W = x.shape
    OC = w.shape[0]
    Ho, Wo = _out_hw(H, W, 3, stride, 1)
    y = np.zeros((OC, Ho, Wo), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ref_lib().vdref_conv3x3_blocked(_fp(x), W, H, IC, _fp(w), OC, _fp(b), int(relu), stride,
                                    _fp(y))
    return y


def ref_conv1x1(x: np.ndarray, w: np.ndarray, stride: int = 1, bias: np.ndarray | None = None,
                relu: bool = False) -> np.ndarray:
    """Reference blocked_conv1x1 (src/directconv.cpp:1510-1522)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w.reshape(w.shape[0], -1), np.float32)
    IC, H, W = x.shape
    OC = w.shape[0]
    Ho, Wo = _out_hw(H, W, 1, stride, 0)
    y = np.zeros((OC, Ho, Wo), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ref_lib().vdref_conv1x1_blocked(_fp(x), W, H, IC, _fp(w), OC, _fp(b), int(relu), stride,
                                    _fp(y))
    return y


def ref_directconv3x3(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Reference NCHW directconv_conv3x3 (stride 1, pad 1, no bias)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    IC, H, W = x.shape
    OC = w.shape[0]
    y = np.zeros((OC, H, W), np.float32)
    ref_lib().vdref_directconv3x3(_fp(x), W, H, IC, _fp(w), OC, _fp(y))
    return y


def ref_winograd3x3(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Reference winograd_conv3x3 (stride 1, pad 1, no bias)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    IC, H, W = x.shape
    OC = w.shape[0]
    y = np.zeros((OC, H, W), np.float32)
    ref_lib().vdref_winograd3x3(_fp(x), W, H, IC, _fp(w), OC, _fp(y))
    return y


# ---------------------------------------------------------------------------
# ResNet34 end to end
# ---------------------------------------------------------------------------
class _DescHolder:
    """Keeps the numpy arrays behind a ResNetDesc alive."""

    def __init__(self, m: dict):
        self.keep = []

        def f(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.float32)
            self.keep.append(a)
            return _fp(a)

        blocks = m["blocks"]
        nb = len(blocks)
        arr = lambda vals: (_f32p * nb)(*vals)  # noqa: E731
        self.c1w = arr([f(b["conv1_w"]) for b in blocks])
        self.c1b = arr([f(b["conv1_b"]) for b in blocks])
        self.c2w = arr([f(b["conv2_w"]) for b in blocks])
        self.c2b = arr([f(b["conv2_b"]) for b in blocks])
        self.dw = arr([f(b.get("down_w")) for b in blocks])
        self.db = arr([f(b.get("down_b")) for b in blocks])
        self.ic = (C.c_int * nb)(*[b["conv1_w"].shape[1] for b in blocks])
        self.oc = (C.c_int * nb)(*[b["conv1_w"].shape[0] for b in blocks])
        self.st = (C.c_int * nb)(*[b["stride"] for b in blocks])
        seg_w = m["seg_w"]
        self.desc = ResNetDesc(
            n_blocks=nb, stem_w=f(m["stem_w"]), stem_b=f(m["stem_b"]),
            stem_oc=m["stem_w"].shape[0], conv1_w=self.c1w, conv1_b=self.c1b,
            conv2_w=self.c2w, conv2_b=self.c2b, down_w=self.dw, down_b=self.db,
            in_ch=self.ic, out_ch=self.oc, stride=self.st, seg_w=f(seg_w), seg_b=f(m["seg_b"]),
            mean_vec=f(m.get("mean_vec")), emb_dim=seg_w.shape[0], pooled_dim=seg_w.shape[1],
            var_eps=float(m.get("var_eps", 1e-8)), l2_normalize=int(m.get("l2_normalize", True)))


def resnet34_embed(model: dict, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """C restatement: feats [n_mels, T] -> (embedding, pre_norm)."""
    h = _DescHolder(model)
    feats = np.ascontiguousarray(feats, np.float32)
    n_mels, T = feats.shape
    D = h.desc.emb_dim
    emb = np.zeros(D, np.float32)
    pre = np.zeros(D, np.float32)
    rc = lib().vdo_resnet34_forward(C.byref(h.desc), _fp(feats), T, n_mels, _fp(emb), _fp(pre))
    if rc != 0:
        raise RuntimeError(f"vdo_resnet34_forward rc={rc}")
    return emb, pre


class RefResNet34:
    """The reference kernels (directconv island) + restated glue, weights registered once."""

    def __init__(self, model: dict):
        self._h = _DescHolder(model)
        self.emb_dim = self._h.desc.emb_dim
        self.handle = ref_lib().vdref_resnet34_new(C.byref(self._h.desc))

    def embed(self, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        feats = np.ascontiguousarray(feats, np.float32)
        n_mels, T = feats.shape
        emb = np.zeros(self.emb_dim, np.float32)
        pre = np.zeros(self.emb_dim, np.float32)
        rc = ref_lib().vdref_resnet34_forward(self.handle, _fp(feats), T, n_mels, _fp(emb),
                                             _fp(pre))
        if rc != 0:
            raise RuntimeError(f"vdref_resnet34_forward rc={rc}")
        return emb, pre


# ---------------------------------------------------------------------------
# ERes2Net end to end
# ---------------------------------------------------------------------------
class ERes2NetDesc(C.Structure):
    _fields_ = [
        ("n_convs", C.c_int), ("w", C.POINTER(_f32p)), ("b", C.POINTER(_f32p)),
        ("ic", _i32p), ("oc", _i32p), ("k", _i32p), ("stride", _i32p),
        ("num_blocks", C.c_int * 4), ("m_channels", C.c_int), ("scale", C.c_int),
        ("relu_clamp", C.c_float), ("seg_w", _f32p), ("seg_b", _f32p), ("emb_dim", C.c_int),
        ("pooled_dim", C.c_int), ("var_eps", C.c_float), ("l2_normalize", C.c_int),
    ]


class _EDescHolder:
    def __init__(self, m: dict):
        self.keep = []

        def f(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, np.float32)
            self.keep.append(a)
            return _fp(a)

        cv = m["convs"]
        n = len(cv)
        self.w = (_f32p * n)(*[f(c["w"]) for c in cv])
        self.b = (_f32p * n)(*[f(c["b"]) for c in cv])
        self.ic = (C.c_int * n)(*[c["w"].shape[1] for c in cv])
        self.oc = (C.c_int * n)(*[c["w"].shape[0] for c in cv])
        self.k = (C.c_int * n)(*[c["w"].shape[2] for c in cv])
        self.st = (C.c_int * n)(*[c["stride"] for c in cv])
        seg_w = m["seg_w"]
        self.desc = ERes2NetDesc(
            n_convs=n, w=self.w, b=self.b, ic=self.ic, oc=self.oc, k=self.k, stride=self.st,
            num_blocks=(C.c_int * 4)(*m["num_blocks"]), m_channels=m["m_channels"],
            scale=m["scale"], relu_clamp=float(m["relu_clamp"]), seg_w=f(seg_w),
            seg_b=f(m["seg_b"]), emb_dim=seg_w.shape[0], pooled_dim=seg_w.shape[1],
            var_eps=float(m["var_eps"]), l2_normalize=int(m.get("l2_normalize", True)))


def eres2net_embed(model: dict, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """C restatement of ERes2NetEncoder::forward_capture -> (embedding, pre_norm)."""
    h = _EDescHolder(model)
    L = lib()
    L.vdo_eres2net_forward.restype = C.c_int
    L.vdo_eres2net_forward.argtypes = [C.POINTER(ERes2NetDesc), _f32p, C.c_int, C.c_int, _f32p,
                                       _f32p]
    feats = np.ascontiguousarray(feats, np.float32)
    n_mels, T = feats.shape
    D = h.desc.emb_dim
    emb = np.zeros(D, np.float32)
    pre = np.zeros(D, np.float32)
    rc = L.vdo_eres2net_forward(C.byref(h.desc), _fp(feats), T, n_mels, _fp(emb), _fp(pre))
    if rc != 0:
        raise RuntimeError(f"vdo_eres2net_forward rc={rc}")
    return emb, pre


class RefERes2Net:
    """The reference's blocked conv kernels + restated ERes2Net glue."""

    def __init__(self, model: dict):
        self._h = _EDescHolder(model)
        L = ref_lib()
        L.vdref_eres2net_new.restype = C.c_void_p
        L.vdref_eres2net_new.argtypes = [C.POINTER(ERes2NetDesc)]
        L.vdref_eres2net_forward.restype = C.c_int
        L.vdref_eres2net_forward.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int, _f32p, _f32p]
        self.emb_dim = self._h.desc.emb_dim
        self.handle = L.vdref_eres2net_new(C.byref(self._h.desc))

    def embed(self, feats: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        feats = np.ascontiguousarray(feats, np.float32)
        n_mels, T = feats.shape
        emb = np.zeros(self.emb_dim, np.float32)
        pre = np.zeros(self.emb_dim, np.float32)
        rc = ref_lib().vdref_eres2net_forward(self.handle, _fp(feats), T, n_mels, _fp(emb),
                                              _fp(pre))
        if rc != 0:
            raise RuntimeError(f"vdref_eres2net_forward rc={rc}")
        return emb, pre


def resample_linear(pcm: np.ndarray, in_sr: int, out_sr: int = 16000) -> np.ndarray:
    pcm = np.ascontiguousarray(pcm, np.float32)
    n_out = lib().vdo_resample_linear(_fp(pcm), len(pcm), in_sr, out_sr, None, 0)
    out = np.zeros(max(n_out, 0), np.float32)
    lib().vdo_resample_linear(_fp(pcm), len(pcm), in_sr, out_sr, _fp(out), len(out))
    return out


def ref_resample_linear(pcm: np.ndarray, in_sr: int, out_sr: int = 16000) -> np.ndarray:
    """The reference's own vd::resample_linear (src/audio_io.cpp:9-23), compiled."""
    L = ref_lib()
    pcm = np.ascontiguousarray(pcm, np.float32)
    n_out = L.vdref_resample_linear(_fp(pcm), len(pcm), in_sr, out_sr, None, 0)
    out = np.zeros(max(n_out, 0), np.float32)
    L.vdref_resample_linear(_fp(pcm), len(pcm), in_sr, out_sr, _fp(out), len(out))
    return out


def ref_load_audio_16k_mono(path) -> np.ndarray:
    """The reference's own vd::load_audio_16k_mono (src/audio_io.cpp:25-38): dr_wav
    decode, f64 channel average, resample to 16 kHz."""
    L = ref_lib()
    p = str(path).encode()
    n = L.vdref_load_audio_16k_mono(p, None, 0)
    if n < 0:
        raise RuntimeError(f"reference could not decode {path}")
    out = np.zeros(n, np.float32)
    L.vdref_load_audio_16k_mono(p, _fp(out), n)
    return out


def ref_drwav_decode(path) -> tuple[np.ndarray, int]:
    """dr_wav's f32 decode (the reference's vendored third_party/dr_wav.h):
    [frames, channels] float32 and the sample rate."""
    L = ref_lib()
    p = str(path).encode()
    ch, sr = C.c_int(0), C.c_int(0)
    frames = L.vdref_drwav_decode_f32(p, None, 0, C.byref(ch), C.byref(sr))
    if frames < 0:
        raise RuntimeError(f"dr_wav could not decode {path}")
    out = np.zeros(frames * ch.value, np.float32)
    L.vdref_drwav_decode_f32(p, _fp(out), len(out), C.byref(ch), C.byref(sr))
    return out.reshape(frames, ch.value), sr.value


def identify(q: np.ndarray, reg: np.ndarray, k: int = 5) -> tuple[np.ndarray, np.ndarray]:
    q = np.ascontiguousarray(q, np.float32)
    reg = np.ascontiguousarray(reg, np.float32)
    nq, dim = q.shape
    idx = np.zeros((nq, k), np.int32)
    sc = np.zeros((nq, k), np.float32)
    lib().vdo_identify(_fp(q), nq, _fp(reg), reg.shape[0], dim, k,
                       idx.ctypes.data_as(_i32p), _fp(sc))
    return idx, sc


# ECAPA-TDNN: numpy restatement (oracle/ecapa.py)
from .ecapa import ecapa_embed  # noqa: E402,F401

# CAM++: numpy restatement (oracle/campplus.py)
from .campplus import campplus_embed  # noqa: E402,F401
