"""Device-side audio ingest (vdb_pcm_ingest, voicedetect_b200_embed_s16_batch): int16
or f32 mono PCM at any rate converted / linearly resampled to f32 16 kHz on the GPU,
replacing the reference's host path (drwav s16 -> f32, resample_linear,
src/audio_io.cpp:9-23). Gates: bitwise equality with the reference's own compiled
resample_linear (oracle/_ref; the oracle's restatement where that library is absent,
itself pinned bitwise to it in tests/test_audio_cpu.py), and embeddings bitwise equal
to the f32 16 kHz path they replace."""
import numpy as np
import pytest

import oracle
import vd_synth

pytestmark = pytest.mark.gpu

RATES = [16000, 8000, 11025, 22050, 44100, 48000]


@pytest.mark.parametrize("rate", RATES)
@pytest.mark.parametrize("dtype", ["s16", "f32"])
def test_ingest_matches_oracle_resample(cuda_lib, rate, dtype):
    import torch
    lens = [rate * 2 + 37, 1, 0, 5, rate // 3, 4 * rate + 1]
    rng = np.random.default_rng(rate)
    clips16 = [vd_synth.make_clip(700 + i, n) if n >= 64 else
               rng.integers(-32768, 32768, n).astype(np.int16) for i, n in enumerate(lens)]
    resample = oracle.ref_resample_linear if oracle.ref_available() else oracle.resample_linear
    want = [resample(vd_synth.clip_f32(c), rate, 16000) for c in clips16]
    dev = torch.device("cuda")
    if dtype == "s16":
        ins = [torch.from_numpy(c.astype(np.int16)).to(dev) for c in clips16]
    else:
        ins = [torch.from_numpy(vd_synth.clip_f32(c)).to(dev) for c in clips16]
    got = cuda_lib.pcm_ingest(ins, rate)
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        g = g.cpu().numpy()
        assert g.shape == w.shape
        assert np.array_equal(g, w)


@pytest.fixture(scope="module")
def resnet(tmp_path_factory, cuda_lib):
    m = vd_synth.resnet34_model(4)
    path = tmp_path_factory.mktemp("ing") / "r.gguf"
    vd_synth.write_resnet_gguf(str(path), m, "f16")
    model = cuda_lib.Model(str(path))
    yield model
    model.close()


def test_s16_batch_equals_f32_batch(resnet):
    lens = [48000, 16000 + 333, 160000, 400 + 160 * 7, 32000]
    c16 = [vd_synth.make_clip(710 + i, n) for i, n in enumerate(lens)]
    a = resnet.embed_batch([vd_synth.clip_f32(c) for c in c16])
    b = resnet.embed_batch_s16(c16)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("rate", [8000, 44100])
def test_resampled_batch_equals_host_resampling(resnet, rate):
    """Device resampling inside the batch call = the host resampling the single-clip
    call does (reference semantics), bit for bit, for f32 and int16 input."""
    c16 = [vd_synth.make_clip(720 + i, n) for i, n in enumerate([rate * 3, rate + 11, rate * 7 // 2])]
    f32 = [vd_synth.clip_f32(c) for c in c16]
    host = resnet.embed_batch([oracle.resample_linear(c, rate, 16000) for c in f32])
    dev_f32 = resnet.embed_batch(f32, sample_rate=rate)
    dev_s16 = resnet.embed_batch_s16(c16, sample_rate=rate)
    assert np.array_equal(host, dev_f32)
    assert np.array_equal(host, dev_s16)
    single = resnet.embed_pcm(f32[0], sample_rate=rate)
    assert float(single @ host[0]) >= 0.999999


def test_s16_batch_rejects_bad_rate(resnet):
    with pytest.raises(Exception):
        resnet.embed_batch_s16([np.zeros(16000, np.int16)], sample_rate=0)
