"""voicedetect_capi_set_devices: one context driving several GPUs. The batch call
shards clips over the GPUs (LPT on length) and must return, in the caller's order,
the same embeddings one GPU computes (the per-clip math does not depend on which
clips share a bucket; only the FC's split-K summation order may differ).

Needs at least two GPUs; skipped otherwise."""
import numpy as np
import pytest

import vd_synth

pytestmark = pytest.mark.gpu


def _cos(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_set_devices_shards_batch(tmp_path, cuda_lib):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    m = vd_synth.resnet34_model(0)
    path = tmp_path / "r.gguf"
    vd_synth.write_resnet_gguf(str(path), m, "f16")
    model = cuda_lib.Model(str(path))
    try:
        lens = [16000 + 1500 * i for i in range(23)]
        clips = [vd_synth.clip_f32(vd_synth.make_clip(800 + i, k)) for i, k in enumerate(lens)]
        one = model.embed_batch(clips)
        model.set_devices(min(n, 4))
        many = model.embed_batch(clips)
        for i in range(len(clips)):
            assert _cos(one[i], many[i]) >= 0.999999, i
        with pytest.raises(cuda_lib.VoiceDetectError, match="n_gpus"):
            model.set_devices(n + 1)
        model.set_devices(1)
        again = model.embed_batch(clips)
        assert np.allclose(again, one, atol=1e-6)
    finally:
        model.close()
