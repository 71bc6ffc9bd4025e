"""ctypes binding of libvoicedetect_b200.so (the B200 engine's C ABI).

Two ABI levels are exposed, mirroring the headers in include/:

* the reference's flat model C ABI, ``voicedetect_capi_*`` (include/voicedetect_capi.h),
  wrapped by :class:`Model`;
* the op-level ABI, ``vdb_*`` (include/vdb_ops.h): the conv / FBank / pooling
  kernels on device buffers, wrapped by :func:`conv` etc. The layout helpers
  (:func:`to_grid` / :func:`from_grid`, :func:`to_phase` / :func:`from_phase`,
  :func:`to_fphase` / :func:`from_fphase`, :func:`to_seq` / :func:`from_seq`,
  :func:`to_tphase` / :func:`from_tphase`) build and read the GRID / PHASE / FPHASE /
  SEQ / TPHASE activation layouts that header defines, with torch (on any device).

There is no CPU fallback: importing works without a GPU, but every compute call
goes to the CUDA library and raises if it is missing or fails.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libvoicedetect_b200.so"

_lib: C.CDLL | None = None


def build() -> None:
    import subprocess
    r = subprocess.run(["make", "-C", str(HERE), "-j8"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("libvoicedetect_b200 build failed:\n" + r.stdout + r.stderr)


class ConvArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int), ("t_out", C.c_int), ("f_out", C.c_int), ("oc", C.c_int),
        ("k0", C.c_int), ("stride0", C.c_int), ("ic0", C.c_int),
        ("x0", C.c_void_p), ("w0", C.c_void_p),
        ("stride1", C.c_int), ("ic1", C.c_int), ("x1", C.c_void_p), ("w1", C.c_void_p),
        ("bias", C.c_void_p), ("residual", C.c_void_p), ("relu", C.c_int),
        ("clamp_hi", C.c_float), ("tvalid", C.c_void_p), ("y", C.c_void_p),
        ("y_phase", C.c_int), ("err", C.c_void_p), ("tile_m", C.c_int), ("halo", C.c_int),
        ("ksplit", C.c_int), ("ldx0", C.c_int), ("ldx1", C.c_int), ("ldy", C.c_int),
        ("y2", C.c_void_p), ("ldr", C.c_int), ("residual2", C.c_void_p), ("ldr2", C.c_int),
        ("act", C.c_int), ("ysum", C.c_void_p), ("ldsum", C.c_int), ("addend", C.c_void_p),
        ("ldaddend", C.c_int), ("y_pad", C.c_int), ("tile_n", C.c_int), ("pair", C.c_int), ("qpack", C.c_int),
        ("w0_scale", C.c_void_p), ("w1_scale", C.c_void_p),
        ("w_scratch", C.c_void_p), ("w_scratch_bytes", C.c_longlong),
    ]


class Conv1dArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int), ("t", C.c_int), ("pad", C.c_int), ("oc", C.c_int),
        ("k0", C.c_int), ("dil0", C.c_int), ("ic0", C.c_int), ("x0", C.c_void_p),
        ("ldx0", C.c_int), ("w0", C.c_void_p), ("ic1", C.c_int), ("x1", C.c_void_p),
        ("ldx1", C.c_int), ("w1", C.c_void_p), ("bias", C.c_void_p), ("clip_bias", C.c_void_p),
        ("bn_scale", C.c_void_p), ("bn_shift", C.c_void_p), ("act", C.c_int), ("relu", C.c_int),
        ("residual", C.c_void_p), ("ldr", C.c_int), ("tvalid", C.c_void_p), ("y", C.c_void_p),
        ("ldy", C.c_int), ("y_f32", C.c_int), ("reflect", C.c_int), ("ysum", C.c_void_p),
        ("ldsum", C.c_int), ("addend", C.c_void_p), ("ldaddend", C.c_int), ("err", C.c_void_p),
        ("tile_m", C.c_int), ("tile_n", C.c_int), ("pair", C.c_int), ("stride0", C.c_int),
        ("gate", C.c_void_p), ("gate_seg", C.c_int), ("gate_nseg", C.c_int),
        ("x_scale", C.c_void_p), ("x_shift", C.c_void_p), ("halo", C.c_int),
    ]


def lib() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing; run `make -C {HERE}`")
        L = C.CDLL(str(LIB_PATH))
        L.vdb_last_error.restype = C.c_char_p
        L.vdb_grid_rows.restype = C.c_longlong
        L.vdb_grid_rows.argtypes = [C.c_int, C.c_int, C.c_int]
        L.vdb_phase_rows.restype = C.c_longlong
        L.vdb_phase_rows.argtypes = [C.c_int, C.c_int, C.c_int]
        L.vdb_conv.restype = C.c_int
        L.vdb_conv.argtypes = [C.POINTER(ConvArgs), C.c_void_p]
        L.vdb_seq_rows.restype = C.c_longlong
        L.vdb_seq_rows.argtypes = [C.c_int, C.c_int, C.c_int]
        L.vdb_conv1d.restype = C.c_int
        L.vdb_conv1d.argtypes = [C.POINTER(Conv1dArgs), C.c_void_p]
        L.vdb_fbank_plan_create.restype = C.c_void_p
        L.vdb_fbank_plan_create.argtypes = [C.c_int] * 5 + [C.c_float] * 3
        L.vdb_fbank_plan_destroy.argtypes = [C.c_void_p]
        L.vdb_fbank.restype = C.c_int
        L.vdb_fbank.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                C.c_void_p, C.c_void_p]
        L.vdb_cmn_stem.restype = C.c_int
        L.vdb_cmn_stem.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                   C.c_void_p]
        L.vdb_cmn_stem_qpack.restype = C.c_int
        L.vdb_cmn_stem_qpack.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p]
        L.vdb_cmn_stem_noalloc.restype = C.c_int
        L.vdb_cmn_stem_noalloc.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                           C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                           C.c_void_p, C.c_void_p]
        L.vdb_pool_embed.restype = C.c_int
        L.vdb_pool_embed.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float,
                                     C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.vdb_add.restype = C.c_int
        L.vdb_add.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                              C.c_longlong, C.c_int, C.c_void_p]
        L.vdb_identify.restype = C.c_int
        L.vdb_identify.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p, C.c_void_p, C.c_void_p]
        # model-level C ABI
        L.voicedetect_capi_abi_version.restype = C.c_int
        L.voicedetect_capi_load.restype = C.c_void_p
        L.voicedetect_capi_load.argtypes = [C.c_char_p]
        L.voicedetect_capi_free.argtypes = [C.c_void_p]
        L.voicedetect_capi_last_error.restype = C.c_char_p
        L.voicedetect_capi_last_error.argtypes = [C.c_void_p]
        L.voicedetect_capi_free_string.argtypes = [C.c_void_p]
        L.voicedetect_capi_free_vec.argtypes = [C.c_void_p]
        L.voicedetect_capi_embed_path.restype = C.c_int
        L.voicedetect_capi_embed_path.argtypes = [C.c_void_p, C.c_char_p,
                                                  C.POINTER(C.POINTER(C.c_float)),
                                                  C.POINTER(C.c_int)]
        L.voicedetect_capi_embed_pcm.restype = C.c_int
        L.voicedetect_capi_embed_pcm.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int,
                                                 C.c_int, C.POINTER(C.POINTER(C.c_float)),
                                                 C.POINTER(C.c_int)]
        L.voicedetect_capi_verify_paths.restype = C.c_int
        L.voicedetect_capi_verify_paths.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p,
                                                    C.c_float, C.POINTER(C.c_float),
                                                    C.POINTER(C.c_int)]
        L.voicedetect_capi_analyze_path_json.restype = C.c_void_p
        L.voicedetect_capi_analyze_path_json.argtypes = [C.c_void_p, C.c_char_p]
        L.voicedetect_capi_embed_pcm_batch.restype = C.c_int
        L.voicedetect_capi_embed_pcm_batch.argtypes = [C.c_void_p,
                                                       C.POINTER(C.POINTER(C.c_float)),
                                                       C.POINTER(C.c_int), C.c_int, C.c_int,
                                                       C.POINTER(C.c_float), C.POINTER(C.c_int)]
        L.voicedetect_b200_embed_s16_batch.restype = C.c_int
        L.voicedetect_b200_embed_s16_batch.argtypes = [C.c_void_p,
                                                       C.POINTER(C.POINTER(C.c_int16)),
                                                       C.POINTER(C.c_int), C.c_int, C.c_int,
                                                       C.POINTER(C.c_float), C.POINTER(C.c_int)]
        L.voicedetect_b200_load_audio_16k_mono.restype = C.c_int
        L.voicedetect_b200_load_audio_16k_mono.argtypes = [C.c_char_p,
                                                           C.POINTER(C.POINTER(C.c_float)),
                                                           C.POINTER(C.c_int)]
        L.voicedetect_b200_audio_error.restype = C.c_char_p
        L.vdb_qpack_rows.restype = C.c_longlong
        L.vdb_qpack_rows.argtypes = [C.c_int, C.c_int, C.c_int]
        L.vdb_qpack_pack_weights.restype = C.c_int
        L.vdb_qpack_pack_weights.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.vdb_resampled_length.restype = C.c_longlong
        L.vdb_resampled_length.argtypes = [C.c_longlong, C.c_int, C.c_int]
        L.vdb_pcm_ingest.restype = C.c_int
        L.vdb_pcm_ingest.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                     C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                     C.c_void_p, C.c_void_p]
        L.voicedetect_capi_identify.restype = C.c_int
        L.voicedetect_capi_identify.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int,
                                                C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int,
                                                C.POINTER(C.c_int), C.POINTER(C.c_float)]
        L.voicedetect_capi_set_devices.restype = C.c_int
        L.voicedetect_capi_set_devices.argtypes = [C.c_void_p, C.c_int]
        L.voicedetect_b200_embed_device.restype = C.c_int
        L.voicedetect_b200_embed_device.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.c_void_p, C.c_int, C.c_void_p,
                                                    C.c_void_p]
        L.voicedetect_b200_set_bucketing.restype = C.c_int
        L.voicedetect_b200_set_bucketing.argtypes = [C.c_void_p, C.c_int, C.c_longlong]
        L.voicedetect_b200_last_launches.restype = C.c_longlong
        L.voicedetect_b200_last_launches.argtypes = [C.c_void_p]
        L.voicedetect_b200_embedding_dim.restype = C.c_int
        L.voicedetect_b200_embedding_dim.argtypes = [C.c_void_p]
        L.voicedetect_b200_sync.restype = C.c_int
        L.voicedetect_b200_sync.argtypes = [C.c_void_p]
        L.voicedetect_b200_profile_convs.restype = C.c_int
        L.voicedetect_b200_profile_convs.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.voicedetect_b200_conv_weight_bytes.restype = C.c_longlong
        L.voicedetect_b200_conv_weight_bytes.argtypes = [C.c_void_p]
        L.voicedetect_b200_release_cache.restype = C.c_int
        L.voicedetect_b200_release_cache.argtypes = [C.c_void_p]
        L.voicedetect_b200_host_register.restype = C.c_int
        L.voicedetect_b200_host_register.argtypes = [C.c_void_p, C.c_size_t]
        L.voicedetect_b200_host_unregister.restype = C.c_int
        L.voicedetect_b200_host_unregister.argtypes = [C.c_void_p]
        L.voicedetect_b200_profile.restype = C.c_int
        L.voicedetect_b200_profile.argtypes = [C.c_void_p, C.c_int]
        L.voicedetect_b200_profile_read.restype = C.c_int
        L.voicedetect_b200_profile_stages.restype = C.c_int
        L.voicedetect_b200_profile_stages.argtypes = [C.c_void_p, C.POINTER(C.c_double), C.c_int]
        L.voicedetect_b200_profile_read.argtypes = [C.c_void_p, C.POINTER(C.c_double),
                                                    C.POINTER(C.c_double),
                                                    C.POINTER(C.c_longlong)]
        _lib = L
    return _lib


class VoiceDetectError(RuntimeError):
    pass


class Model:
    """A loaded speaker model behind the reference-compatible C ABI
    (voicedetect_capi_*). Mirrors vd::Model (src/model.hpp): embed_path,
    embed_pcm, verify_paths, plus the additive batch / identify calls."""

    def __init__(self, gguf_path: str):
        self._L = lib()
        self.ctx = self._L.voicedetect_capi_load(str(gguf_path).encode())
        if not self.ctx:
            raise VoiceDetectError(f"voicedetect_capi_load failed for {gguf_path}")
        self.dim = self._L.voicedetect_b200_embedding_dim(self.ctx)

    def close(self) -> None:
        if getattr(self, "ctx", None):
            self._L.voicedetect_capi_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return self._L.voicedetect_capi_last_error(self.ctx).decode()

    def _vec(self, rc, p, d):
        import numpy as np
        if rc != 0:
            raise VoiceDetectError(self.last_error())
        out = np.ctypeslib.as_array(p, shape=(d.value,)).copy()
        self._L.voicedetect_capi_free_vec(C.cast(p, C.c_void_p))
        return out

    def embed_pcm(self, pcm, sample_rate: int = 16000):
        import numpy as np
        pcm = np.ascontiguousarray(pcm, dtype=np.float32)
        p = C.POINTER(C.c_float)()
        d = C.c_int(0)
        rc = self._L.voicedetect_capi_embed_pcm(self.ctx, pcm.ctypes.data_as(C.POINTER(C.c_float)),
                                                len(pcm), sample_rate, C.byref(p), C.byref(d))
        return self._vec(rc, p, d)

    def embed_path(self, path: str):
        p = C.POINTER(C.c_float)()
        d = C.c_int(0)
        rc = self._L.voicedetect_capi_embed_path(self.ctx, str(path).encode(), C.byref(p),
                                                 C.byref(d))
        return self._vec(rc, p, d)

    def verify_paths(self, a: str, b: str, threshold: float = 0.25):
        dist = C.c_float(0)
        ok = C.c_int(0)
        rc = self._L.voicedetect_capi_verify_paths(self.ctx, str(a).encode(), str(b).encode(),
                                                   threshold, C.byref(dist), C.byref(ok))
        if rc != 0:
            raise VoiceDetectError(self.last_error())
        return float(dist.value), bool(ok.value)

    def embed_batch(self, clips, sample_rate: int = 16000):
        import numpy as np
        arrs = [np.ascontiguousarray(c, dtype=np.float32) for c in clips]
        n = len(arrs)
        addr = np.fromiter((a.__array_interface__["data"][0] for a in arrs), np.uint64, n)
        lens = np.fromiter((len(a) for a in arrs), np.int32, n)
        ptrs = addr.ctypes.data_as(C.POINTER(C.POINTER(C.c_float)))
        ns = lens.ctypes.data_as(C.POINTER(C.c_int))
        out = np.zeros((n, self.dim), np.float32)
        d = C.c_int(0)
        rc = self._L.voicedetect_capi_embed_pcm_batch(self.ctx, ptrs, ns, n, sample_rate,
                                                      out.ctypes.data_as(C.POINTER(C.c_float)),
                                                      C.byref(d))
        if rc != 0:
            raise VoiceDetectError(self.last_error())
        return out

    def embed_batch_s16(self, clips, sample_rate: int = 16000):
        """int16 mono clips (voicedetect_b200_embed_s16_batch): converted and, at other
        rates, resampled on the GPU."""
        import numpy as np
        arrs = [np.ascontiguousarray(c, dtype=np.int16) for c in clips]
        n = len(arrs)
        addr = np.fromiter((a.__array_interface__["data"][0] for a in arrs), np.uint64, n)
        lens = np.fromiter((len(a) for a in arrs), np.int32, n)
        ptrs = addr.ctypes.data_as(C.POINTER(C.POINTER(C.c_int16)))
        ns = lens.ctypes.data_as(C.POINTER(C.c_int))
        out = np.zeros((n, self.dim), np.float32)
        d = C.c_int(0)
        rc = self._L.voicedetect_b200_embed_s16_batch(self.ctx, ptrs, ns, n, sample_rate,
                                                      out.ctypes.data_as(C.POINTER(C.c_float)),
                                                      C.byref(d))
        if rc != 0:
            raise VoiceDetectError(self.last_error())
        return out

    def identify(self, queries, registry, k: int = 5):
        import numpy as np
        q = np.ascontiguousarray(queries, np.float32)
        r = np.ascontiguousarray(registry, np.float32)
        idx = np.zeros((q.shape[0], k), np.int32)
        sc = np.zeros((q.shape[0], k), np.float32)
        rc = self._L.voicedetect_capi_identify(self.ctx, q.ctypes.data_as(C.POINTER(C.c_float)),
                                               q.shape[0], r.ctypes.data_as(C.POINTER(C.c_float)),
                                               r.shape[0], q.shape[1], k,
                                               idx.ctypes.data_as(C.POINTER(C.c_int)),
                                               sc.ctypes.data_as(C.POINTER(C.c_float)))
        if rc != 0:
            raise VoiceDetectError(self.last_error())
        return idx, sc

    def set_devices(self, n_gpus: int) -> None:
        """Use n_gpus GPUs (the batch call shards clips over them)."""
        if self._L.voicedetect_capi_set_devices(self.ctx, n_gpus) != 0:
            raise VoiceDetectError(self.last_error())

    def set_bucketing(self, max_clips: int, max_frames: int) -> None:
        if self._L.voicedetect_b200_set_bucketing(self.ctx, max_clips, max_frames) != 0:
            raise VoiceDetectError(self.last_error())

    def embed_device(self, d_pcm, offsets, n_samples, d_out, stream=None) -> None:
        """Device-resident batch: d_pcm / d_out torch CUDA tensors; offsets /
        n_samples host int sequences."""
        n = len(n_samples)
        offs = (C.c_longlong * n)(*[int(o) for o in offsets])
        ns = (C.c_int * n)(*[int(v) for v in n_samples])
        rc = self._L.voicedetect_b200_embed_device(self.ctx, d_pcm.data_ptr(), offs, ns, n,
                                                   d_out.data_ptr(),
                                                   C.c_void_p(stream) if stream else None)
        if rc != 0:
            raise VoiceDetectError(self.last_error())

    def last_launches(self) -> int:
        return int(self._L.voicedetect_b200_last_launches(self.ctx))

    def sync(self) -> None:
        if self._L.voicedetect_b200_sync(self.ctx) != 0:
            raise VoiceDetectError(self.last_error())

    def profile_convs(self) -> list[dict]:
        """The conv launches of the last profile read (profile_read), in order."""
        n = self._L.voicedetect_b200_profile_convs(self.ctx, None, 0)
        if n <= 0:
            return []
        buf = (C.c_double * (12 * n))()
        self._L.voicedetect_b200_profile_convs(self.ctx, buf, n)
        keys = ("ms", "flops", "ic", "oc", "k", "stride", "f_out", "t_out", "batch", "ic1",
                "res", "qpack")
        return [{k: (buf[12 * i + j] if j < 2 else int(buf[12 * i + j]))
                 for j, k in enumerate(keys)} for i in range(n)]

    @property
    def conv_weight_bytes(self) -> int:
        """Device bytes of the ResNet block conv weights (q8_0 stays q8_0)."""
        return int(self._L.voicedetect_b200_conv_weight_bytes(self.ctx))

    def release_cache(self) -> None:
        """Drops the captured CUDA graphs and the workspace (weights stay resident)."""
        if self._L.voicedetect_b200_release_cache(self.ctx) != 0:
            raise VoiceDetectError(self.last_error())

    def profile(self, enable: bool) -> None:
        self._L.voicedetect_b200_profile(self.ctx, int(enable))

    def profile_read(self):
        """-> (conv_ms, conv_flops, conv_launches) since the previous read."""
        ms, fl, n = C.c_double(0), C.c_double(0), C.c_longlong(0)
        if self._L.voicedetect_b200_profile_read(self.ctx, C.byref(ms), C.byref(fl),
                                                 C.byref(n)) != 0:
            raise VoiceDetectError(self.last_error())
        return ms.value, fl.value, n.value

    def profile_stages(self):
        """-> {conv, fbank, stem, pool, other}: ms per stage of the last profile_read."""
        v = (C.c_double * 5)()
        if self._L.voicedetect_b200_profile_stages(self.ctx, v, 5) != 0:
            raise VoiceDetectError(self.last_error())
        return dict(zip(("conv", "fbank", "stem", "pool", "other"), list(v)))


def last_error() -> str:
    return lib().vdb_last_error().decode()


def host_register(arr) -> bool:
    """Page-lock a contiguous numpy array in place (voicedetect_b200_host_register), so
    the batch calls copy clips stored in it straight to the GPU. Returns False, with
    the reason in last_error(), where the host refuses; the array stays usable."""
    return lib().voicedetect_b200_host_register(arr.ctypes.data, arr.nbytes) == 0


def host_unregister(arr) -> None:
    """Undo host_register(arr) (before the array is freed)."""
    _check(lib().voicedetect_b200_host_unregister(arr.ctypes.data), "host_unregister")


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {last_error()}")


# ---------------------------------------------------------------------------
# Layout helpers (torch, on device). x: (B, C, F, T) in torch NCHW terms with
# H = freq, W = time, matching the reference's ggml [W=T, H=F, C, N].
# ---------------------------------------------------------------------------
def out_extent(n: int, stride: int) -> int:
    return (n - 1) // stride + 1


def to_grid(x, tvalid=None):
    """(B, C, F, T) float -> GRID f16 tensor of shape (B*(T+2)*(F+2), C)."""
    import torch
    B, Cc, F, T = x.shape
    g = torch.zeros(B, T + 2, F + 2, Cc, dtype=torch.float16, device=x.device)
    g[:, 1:T + 1, 1:F + 1, :] = x.permute(0, 3, 2, 1).to(torch.float16)
    if tvalid is not None:
        for b, tv in enumerate(tvalid):
            g[b, 1 + int(tv):, :, :] = 0
    return g.reshape(B * (T + 2) * (F + 2), Cc).contiguous()


def from_grid(g, B: int, C_: int, F: int, T: int):
    """GRID (rows, C) -> (B, C, F, T) float32 (valid interior only)."""
    x = g.reshape(B, T + 2, F + 2, C_)[:, 1:T + 1, 1:F + 1, :]
    return x.permute(0, 3, 2, 1).float().contiguous()


def qpack_width(F: int) -> int:
    """QPACK rows per time step: ceil((F + 2) / 4)."""
    return (F + 2 + 3) // 4


def to_qpack(x, tvalid=None):
    """(B, 32, F, T) -> QPACK f16 tensor (B*(T+2)*Wq, 128): four padded frequency
    pixels per row (include/vdb_ops.h, vdb_qpack_rows)."""
    import torch
    B, Cc, F, T = x.shape
    assert Cc == 32
    Wq = qpack_width(F)
    g = torch.zeros(B, T + 2, 4 * Wq, Cc, dtype=torch.float16, device=x.device)
    g[:, 1:T + 1, 1:F + 1, :] = x.permute(0, 3, 2, 1).to(torch.float16)
    if tvalid is not None:
        for b, tv in enumerate(tvalid):
            g[b, 1 + int(tv):, :, :] = 0
    return g.reshape(B * (T + 2) * Wq, 4 * Cc).contiguous()


def from_qpack(q, B: int, F: int, T: int, interior: bool = True):
    """QPACK (rows, 128) -> (B, 32, F, T) float32 (valid interior), or with
    interior=False the whole padded (B, 32, 4*Wq, T+2) grid."""
    Wq = qpack_width(F)
    g = q.reshape(B, T + 2, 4 * Wq, 32)
    if interior:
        g = g[:, 1:T + 1, 1:F + 1, :]
    return g.permute(0, 3, 2, 1).float().contiguous()


def qpack_weights(w_taps):
    """f16 [32][9][32] conv weight (pack_conv_weight) -> the packed [1152][32] weight of
    a QPACK conv (vdb_qpack_pack_weights, on the device)."""
    import torch
    out = torch.empty(1152, 32, dtype=torch.float16, device=w_taps.device)
    s = torch.cuda.current_stream().cuda_stream
    _check(lib().vdb_qpack_pack_weights(w_taps.contiguous().data_ptr(), out.data_ptr(),
                                        C.c_void_p(s)), "vdb_qpack_pack_weights")
    return out


def qpack_rows():
    """Source row (oc * 9 + tap) of each of the 1152 rows of the QPACK packed weight
    (the layout vdb_qpack_pack_weights writes)."""
    src = []
    for kt in range(3):
        for u in range(-1, 5):
            for j in range(max(0, u - 1), min(3, u + 1) + 1):
                src += [oc * 9 + kt * 3 + (u - j + 1) for oc in range(32)]
    return src


def qpack_q8(q, d):
    """q8_0 operands of a 32 -> 32 conv ((32, 9, 32) int8, (9, 32) block-major f16
    scales, as q8_planes returns them) -> the QPACK packing of both ((1152, 32) int8,
    (1152,) f16: one scale per packed row)."""
    import torch
    idx = torch.tensor(qpack_rows(), device=q.device)
    return q.reshape(288, 32)[idx].contiguous(), d.t().reshape(288)[idx].contiguous()


def to_phase(x, tvalid=None):
    """(B, C, F, T) -> PHASE f16 tensor (4*B*(To+2)*(Fo+2), C) for a stride-2 consumer."""
    import torch
    B, Cc, F, T = x.shape
    To, Fo = out_extent(T, 2), out_extent(F, 2)
    pad = torch.zeros(B, T + 2, F + 2, Cc, dtype=torch.float16, device=x.device)
    pad[:, 1:T + 1, 1:F + 1, :] = x.permute(0, 3, 2, 1).to(torch.float16)
    if tvalid is not None:
        for b, tv in enumerate(tvalid):
            pad[b, 1 + int(tv):, :, :] = 0
    out = torch.zeros(4, B, To + 2, Fo + 2, Cc, dtype=torch.float16, device=x.device)
    for pt in range(2):
        for pf in range(2):
            src = pad[:, pt::2, pf::2, :]
            nt, nf = src.shape[1], src.shape[2]
            out[2 * pt + pf, :, 1:1 + nt, 1:1 + nf, :] = src
    return out.reshape(-1, Cc).contiguous()


def from_phase(p, B: int, C_: int, F: int, T: int):
    """PHASE tensor of a (B, C, F, T) activation -> (B, C, F, T) float32."""
    import torch
    To, Fo = out_extent(T, 2), out_extent(F, 2)
    pl = p.reshape(4, B, To + 2, Fo + 2, C_)
    pad = torch.zeros(B, T + 2, F + 2, C_, dtype=p.dtype, device=p.device)
    for pt in range(2):
        for pf in range(2):
            nt = len(range(pt, T + 2, 2))
            nf = len(range(pf, F + 2, 2))
            pad[:, pt::2, pf::2, :] = pl[2 * pt + pf, :, 1:1 + nt, 1:1 + nf, :]
    return pad[:, 1:T + 1, 1:F + 1, :].permute(0, 3, 2, 1).float().contiguous()


def to_fphase(x, tvalid=None):
    """(B, C, F, T) -> FPHASE f16 tensor (2*B*(T+2)*(Fo+2), C) for a consumer that
    strides 2 along frequency only."""
    import torch
    B, Cc, F, T = x.shape
    Fo = out_extent(F, 2)
    pad = torch.zeros(B, T + 2, F + 2, Cc, dtype=torch.float16, device=x.device)
    pad[:, 1:T + 1, 1:F + 1, :] = x.permute(0, 3, 2, 1).to(torch.float16)
    if tvalid is not None:
        for b, tv in enumerate(tvalid):
            pad[b, 1 + int(tv):, :, :] = 0
    out = torch.zeros(2, B, T + 2, Fo + 2, Cc, dtype=torch.float16, device=x.device)
    for pf in range(2):
        src = pad[:, :, pf::2, :]
        out[pf, :, :, 1:1 + src.shape[2], :] = src
    return out.reshape(-1, Cc).contiguous()


def from_fphase(p, B: int, C_: int, F: int, T: int):
    """FPHASE tensor of a (B, C, F, T) activation -> (B, C, F, T) float32."""
    import torch
    Fo = out_extent(F, 2)
    pl = p.reshape(2, B, T + 2, Fo + 2, C_)
    pad = torch.zeros(B, T + 2, F + 2, C_, dtype=p.dtype, device=p.device)
    for pf in range(2):
        nf = len(range(pf, F + 2, 2))
        pad[:, :, pf::2, :] = pl[pf, :, :, 1:1 + nf, :]
    return pad[:, 1:T + 1, 1:F + 1, :].permute(0, 3, 2, 1).float().contiguous()


def from_tphase(tp, B: int, C_: int, T: int, pad: int):
    """TPHASE (2*B*(To+2*pad), C) of a T-frame sequence -> (B, C, T) float32."""
    To = out_extent(T, 2)
    pl = tp.reshape(2, B, To + 2 * pad, C_)
    out = pl.new_zeros(B, T, C_)
    out[:, 0::2] = pl[0, :, pad:pad + len(range(0, T, 2))]
    out[:, 1::2] = pl[1, :, pad:pad + len(range(1, T, 2))]
    return out.permute(0, 2, 1).float().contiguous()


def to_tphase(x, pad: int, tvalid=None):
    """(B, C, T) float -> TPHASE f16 (2*B*(To+2*pad), C), To = (T-1)//2+1, zero
    outside each clip's valid frames."""
    import torch
    B, Cc, T = x.shape
    To = out_extent(T, 2)
    out = torch.zeros(2, B, To + 2 * pad, Cc, dtype=torch.float16, device=x.device)
    for b in range(B):
        tv = T if tvalid is None else int(tvalid[b])
        xb = x[b, :, :tv].t().to(torch.float16)
        ev, od = xb[0::2], xb[1::2]
        out[0, b, pad:pad + ev.shape[0]] = ev
        out[1, b, pad:pad + od.shape[0]] = od
    return out.reshape(-1, Cc).contiguous()


def q8_planes(w):
    """f16/f32 weights with input channels last (a multiple of 32), e.g. the packed
    (OC, k*k, IC) conv weight -> the q8_0 operands of vdb_conv: the gguf q8_0 rule
    d = max|w| / 127 per block of 32, q = round(w / d). Returns (q, d, w16): q int8 in
    w's shape, d the f16 scales block-major (K / 32, OC) (the w_scale layout), and
    w16 = f16(q * d), the f16 weights the kernel expands them to."""
    import torch
    wf = w.float()
    blk = wf.reshape(*wf.shape[:-1], wf.shape[-1] // 32, 32)
    d = (blk.abs().amax(-1) / 127.0).to(torch.float16)
    df = d.float()
    q = torch.where(df[..., None] > 0, torch.round(blk / df[..., None].clamp_min(1e-30)),
                    torch.zeros_like(blk)).clamp(-127, 127).to(torch.int8)
    w16 = (q.float() * df[..., None]).to(torch.float16).reshape(wf.shape)
    d_t = d.reshape(wf.shape[0], -1).t().contiguous()
    return q.reshape(wf.shape).contiguous(), d_t, w16.contiguous()


def pack_conv_weight(w):
    """torch (OC, IC, KF, KT) -> f16 (OC, KT*KF, IC) (tap = kt*k + kf)."""
    OC, IC, KF, KT = w.shape
    return w.permute(0, 3, 2, 1).reshape(OC, KT * KF, IC).to(
        __import__("torch").float16).contiguous()


def _ld(t):
    """Row pitch in elements of a 2-D (rows, C) tensor or channel-slice view of one."""
    return int(t.stride(0)) if t is not None and t.dim() == 2 else 0


def _ptr(t):
    return t.data_ptr() if t is not None else None


def conv(x0, w0, bias, tvalid, *, batch, t_out, f_out, oc, k0=3, stride0=1, ic0=None,
         x1=None, w1=None, stride1=1, ic1=None, residual=None, relu=False, clamp_hi=0.0,
         y=None, y_phase=False, err=None, stream=None, tile_m=0, halo=0, ksplit=0,
         y2=None, residual2=None, act=0, ysum=None, addend=None, y_pad=0, tile_n=0, pair=0,
         qpack=False, w0_scale=None, w1_scale=None, w_scratch=None):
    """vdb_conv on device tensors. x0/x1/residual/residual2/y are f16 GRID or PHASE
    tensors of shape (rows, C), or channel-slice views of wider ones (x[:, c0:c1]:
    the row pitch is taken from the view's stride); y2 is an extra PHASE output,
    w0 f16 (OC, k*k, IC), w1 f16 (OC, IC1), bias f32 (OC,) or None, tvalid int32 (B,).
    act: 0 = [+residual] then relu/clamp, 1 = SiLU, 2 = attentional fusion
    (residual + residual2) + tanh(acc + bias) * (residual - residual2).
    ysum / addend: optional second GRID output ysum = f16(y + addend).
    stride 3 / y_phase 2: the frequency-only stride-2 input / output (FPHASE);
    y_phase 3: a TPHASE output for a time-stride-2 1-D consumer with y_pad padding
    rows, shaped (2*B*(To+2*y_pad), f_out*oc)."""
    import torch
    if y is None and qpack:
        y = torch.empty(lib().vdb_phase_rows(batch, t_out, f_out) if y_phase
                        else lib().vdb_qpack_rows(batch, t_out, f_out), 32 if y_phase else 128,
                        dtype=torch.float16, device=x0.device)
    if y is None:
        yp = int(y_phase)
        if yp == 3:
            To = out_extent(t_out, 2)
            y = torch.zeros(2 * batch * (To + 2 * y_pad), f_out * oc, dtype=torch.float16,
                            device=x0.device)
        else:
            rows = (lib().vdb_phase_rows(batch, t_out, f_out) if yp == 1
                    else 2 * batch * (t_out + 2) * (out_extent(f_out, 2) + 2) if yp == 2
                    else lib().vdb_grid_rows(batch, t_out, f_out))
            y = torch.empty(rows, oc, dtype=torch.float16, device=x0.device)
    ldy = 0 if (int(y_phase) == 3 or qpack) else _ld(y)
    if w_scratch is None and (w0_scale is not None or w1_scale is not None):
        # room for the f16 expansion of both segments' weights (used if they stream)
        n = w0.numel() + (w1.numel() if (w1 is not None and w1_scale is not None) else 0)
        w_scratch = torch.empty(2 * n + 512, dtype=torch.uint8, device=x0.device)
    a = ConvArgs(batch=batch, t_out=t_out, f_out=f_out, oc=oc, k0=k0, stride0=stride0,
                 ic0=ic0 if ic0 is not None else x0.shape[1], x0=x0.data_ptr(),
                 w0=w0.data_ptr(), stride1=stride1,
                 ic1=(ic1 if ic1 is not None else (x1.shape[1] if x1 is not None else 0)),
                 x1=_ptr(x1), w1=_ptr(w1), bias=_ptr(bias), residual=_ptr(residual),
                 relu=int(relu), clamp_hi=float(clamp_hi), tvalid=tvalid.data_ptr(),
                 y=y.data_ptr(), y_phase=int(y_phase), err=_ptr(err), tile_m=tile_m,
                 halo=halo, ksplit=ksplit, ldx0=_ld(x0), ldx1=_ld(x1), ldy=ldy,
                 y2=_ptr(y2), ldr=_ld(residual), residual2=_ptr(residual2),
                 ldr2=_ld(residual2), act=int(act), ysum=_ptr(ysum), ldsum=_ld(ysum),
                 addend=_ptr(addend), ldaddend=_ld(addend), y_pad=int(y_pad),
                 tile_n=int(tile_n), pair=int(pair), qpack=int(bool(qpack)),
                 w0_scale=_ptr(w0_scale), w1_scale=_ptr(w1_scale),
                 w_scratch=_ptr(w_scratch),
                 w_scratch_bytes=(w_scratch.numel() * w_scratch.element_size()
                                  if w_scratch is not None else 0))
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    _check(lib().vdb_conv(C.byref(a), C.c_void_p(s)), "vdb_conv")
    return y


# ---------------------------------------------------------------------------
# 1-D (TDNN) convs on the SEQ layout: x (B, C, T) <-> (B*(T+2*pad), C) f16 rows
# ---------------------------------------------------------------------------
def to_seq(x, pad: int, tvalid=None, reflect: bool = True):
    """(B, C, T) float -> SEQ f16 (B*(T+2*pad), C). With reflect, the pad rows on
    either side of each clip's valid frames hold their reflection; other rows 0."""
    import torch
    B, Cc, T = x.shape
    s = torch.zeros(B, T + 2 * pad, Cc, dtype=torch.float16, device=x.device)
    for b in range(B):
        tv = T if tvalid is None else int(tvalid[b])
        xb = x[b, :, :tv].t().to(torch.float16)
        s[b, pad:pad + tv] = xb
        if reflect:
            for j in range(1, pad + 1):
                if j < tv:
                    s[b, pad - j] = xb[j]
                    s[b, pad + tv - 1 + j] = xb[tv - 1 - j]
    return s.reshape(B * (T + 2 * pad), Cc).contiguous()


def from_seq(s, B: int, C_: int, T: int, pad: int):
    """SEQ (rows, C) -> (B, C, T) float32 (frame slots 0..T-1)."""
    return s.reshape(B, T + 2 * pad, C_)[:, pad:pad + T, :].permute(0, 2, 1).float().contiguous()


def pack_conv1d_weight(w):
    """torch (OC, IC, K) -> f16 (OC, K, IC)."""
    return w.permute(0, 2, 1).to(__import__("torch").float16).contiguous()


def conv1d(x0, w0, bias, tvalid, *, batch, t, pad, oc, k0=1, dil0=1, ic0=None, x1=None,
           w1=None, ic1=None, bn_scale=None, bn_shift=None, clip_bias=None, act=0, relu=False,
           residual=None, y=None, y_f32=False, reflect=False, ysum=None, addend=None, err=None,
           stream=None, tile_m=0, tile_n=0, pair=0, stride0=1, gate=None, gate_seg=0,
           gate_nseg=0, x_scale=None, x_shift=None, halo=0):
    """vdb_conv1d on device tensors: x0/x1/residual/y/ysum/addend are SEQ tensors
    (rows, C) or channel-slice views of wider ones; w0 f16 (OC, K, IC), w1 f16
    (OC, IC1); bias / bn_scale / bn_shift f32 (OC,); clip_bias f32 (B, OC).
    act: 0 = acc + bias [+ residual] (then ReLU if relu), 1 = SiLU,
    3 = BN(ReLU(acc + bias + clip_bias)), 4 = tanh of act 3, 5 = (acc + bias) *
    gate[b, t // gate_seg] with gate f32 (B, gate_nseg, OC). reflect: 0 / False valid
    frames only, 1 / True reflection rows, 2 zero padding. stride0 2: x0 is TPHASE.
    x_scale / x_shift f32 (IC,): the 1x1 conv reads max(x0 * x_scale + x_shift, 0)."""
    import torch
    if y is None:
        rows = lib().vdb_seq_rows(batch, t, pad)
        y = torch.empty(rows, oc, dtype=torch.float32 if y_f32 else torch.float16,
                        device=x0.device)
    a = Conv1dArgs(batch=batch, t=t, pad=pad, oc=oc, k0=k0, dil0=dil0,
                   ic0=ic0 if ic0 is not None else x0.shape[1], x0=x0.data_ptr(), ldx0=_ld(x0),
                   w0=w0.data_ptr(),
                   ic1=(ic1 if ic1 is not None else (x1.shape[1] if x1 is not None else 0)),
                   x1=_ptr(x1), ldx1=_ld(x1), w1=_ptr(w1), bias=_ptr(bias),
                   clip_bias=_ptr(clip_bias), bn_scale=_ptr(bn_scale), bn_shift=_ptr(bn_shift),
                   act=int(act), relu=int(relu), residual=_ptr(residual), ldr=_ld(residual),
                   tvalid=tvalid.data_ptr(), y=y.data_ptr(), ldy=_ld(y), y_f32=int(y_f32),
                   reflect=int(reflect), ysum=_ptr(ysum), ldsum=_ld(ysum), addend=_ptr(addend),
                   ldaddend=_ld(addend), err=_ptr(err), tile_m=tile_m, tile_n=tile_n,
                   pair=pair, stride0=int(stride0), gate=_ptr(gate), gate_seg=int(gate_seg),
                   gate_nseg=int(gate_nseg), x_scale=_ptr(x_scale), x_shift=_ptr(x_shift),
                   halo=int(halo))
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    _check(lib().vdb_conv1d(C.byref(a), C.c_void_p(s)), "vdb_conv1d")
    return y


def pcm_ingest(clips, sample_rate: int, out_rate: int = 16000):
    """vdb_pcm_ingest on device tensors: list of 1-D int16 or f32 torch tensors (one
    dtype) -> list of f32 tensors at out_rate."""
    import torch
    dev = clips[0].device
    s16 = clips[0].dtype == torch.int16
    n_in = [int(c.numel()) for c in clips]
    n_out = [int(lib().vdb_resampled_length(n, sample_rate, out_rate)) for n in n_in]
    cat = torch.cat(clips)
    in_off = torch.tensor([0] + list(__import__("itertools").accumulate(n_in))[:-1],
                          dtype=torch.int64, device=dev)
    out_off_l = [0] + list(__import__("itertools").accumulate(n_out))[:-1]
    out = torch.zeros(max(sum(n_out), 1), dtype=torch.float32, device=dev)
    a = torch.tensor(n_in, dtype=torch.int32, device=dev)
    b = torch.tensor(n_out, dtype=torch.int32, device=dev)
    oo = torch.tensor(out_off_l, dtype=torch.int64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    _check(lib().vdb_pcm_ingest(cat.data_ptr(), 1 if s16 else 0, in_off.data_ptr(), a.data_ptr(),
                                len(clips), sample_rate, out_rate, oo.data_ptr(), b.data_ptr(),
                                max(n_out), out.data_ptr(), C.c_void_p(s)), "vdb_pcm_ingest")
    return [out[o:o + n] for o, n in zip(out_off_l, n_out)]


def add(a, b, y=None, stream=None):
    """vdb_add: y = a + b on (rows, C) f16 tensors or channel-slice views."""
    import torch
    rows, Cc = a.shape
    if y is None:
        y = torch.empty(rows, Cc, dtype=torch.float16, device=a.device)
    s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
    _check(lib().vdb_add(a.data_ptr(), _ld(a), b.data_ptr(), _ld(b), y.data_ptr(), _ld(y),
                         rows, Cc, C.c_void_p(s)), "vdb_add")
    return y


def load_audio_16k_mono(path: str):
    """Decode a WAV file and resample it to 16 kHz mono through the library's audio
    front door (voicedetect_b200_load_audio_16k_mono; host code, no GPU needed).
    Returns a float32 numpy array."""
    import numpy as np
    L = lib()
    buf = C.POINTER(C.c_float)()
    n = C.c_int(0)
    if L.voicedetect_b200_load_audio_16k_mono(str(path).encode(), C.byref(buf), C.byref(n)) != 0:
        raise RuntimeError(L.voicedetect_b200_audio_error().decode())
    try:
        return np.ctypeslib.as_array(buf, shape=(n.value,)).copy() if n.value else \
            np.zeros(0, np.float32)
    finally:
        L.voicedetect_capi_free_vec(buf)
