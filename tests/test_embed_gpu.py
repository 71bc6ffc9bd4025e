"""End-to-end GPU parity through the reference-compatible C ABI
(voicedetect_capi_*): PCM -> FBank -> CMN+stem -> tensor-core ResNet34 ->
TSTP+FC+L2, against the CPU oracle on the same seeded inputs.

Oracle: oracle/vd_oracle.c restated ResNet34 forward, pinned bit-exact to the
reference's own kernels in tests/test_oracle.py. Gates (BASELINE / the reference's
docs/parity.md): embedding cosine >= 0.9999 and identical verify verdicts.
"""
import numpy as np
import pytest

import oracle
import vd_synth

pytestmark = pytest.mark.gpu

COS_TOL = 0.9999


def _cos(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.fixture(scope="module")
def resnet(tmp_path_factory, cuda_lib):
    m = vd_synth.resnet34_model(0)
    path = tmp_path_factory.mktemp("m") / "resnet34_f32.gguf"
    vd_synth.write_resnet_gguf(str(path), m, "f32")
    model = cuda_lib.Model(str(path))
    yield m, model
    model.close()


def _oracle_embed(m, pcm):
    return oracle.resnet34_embed(m, oracle.fbank(pcm))[0]


def test_embed_pcm_matches_oracle(resnet):
    m, model = resnet
    pcm = vd_synth.clip_f32(vd_synth.make_clip(1, 48000))  # config 0: 3.0 s, T = 298
    got = model.embed_pcm(pcm)
    want = _oracle_embed(m, pcm)
    assert got.shape == (256,)
    assert abs(float(np.linalg.norm(got)) - 1.0) < 1e-3  # tests/test_embed.cpp gate
    assert _cos(got, want) >= COS_TOL


def test_batch_ragged_matches_oracle(resnet):
    m, model = resnet
    lens = [48000, 16000, 31999, 401 + 160 * 7, 80000, 20000]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(100 + i, n)) for i, n in enumerate(lens)]
    got = model.embed_batch(clips)
    for i, c in enumerate(clips):
        assert _cos(got[i], _oracle_embed(m, c)) >= COS_TOL, i
    # one clip alone equals the same clip inside a ragged batch
    single = model.embed_pcm(clips[3])
    assert _cos(single, got[3]) >= 0.99999


def test_bucketing_splits_are_exact(resnet):
    m, model = resnet
    lens = [16000 + 1600 * i for i in range(9)]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(300 + i, n)) for i, n in enumerate(lens)]
    full = model.embed_batch(clips)
    model.set_bucketing(2, 10_000_000)  # force many small buckets
    try:
        split = model.embed_batch(clips)
    finally:
        model.set_bucketing(512, 262144)
    for i in range(len(clips)):
        assert _cos(full[i], split[i]) >= 0.99999


def test_odd_staging_capacity_both_slots(resnet, tmp_path, cuda_lib):
    """A fresh engine whose first bucket holds an odd number of clips (65, above the
    64-clip floor) sizes its two per-bucket metadata slots from that count; four
    buckets alternate between the slots, so the staging kernel reads int64 clip
    offsets from both. Both the device-resident and the host-PCM call must give the
    same embeddings as the shared engine's one-bucket batch."""
    import torch
    m, model = resnet
    path = tmp_path / "resnet34_f32.gguf"
    vd_synth.write_resnet_gguf(str(path), m, "f32")
    fresh = cuda_lib.Model(str(path))
    try:
        lens = [8000 + 160 * (i % 7) for i in range(200)]
        clips = [vd_synth.clip_f32(vd_synth.make_clip(900 + i, n)) for i, n in enumerate(lens)]
        want = model.embed_batch(clips)
        fresh.set_bucketing(65, 10_000_000)
        pcm = np.concatenate(clips)
        offs = np.zeros(len(lens), np.int64)
        offs[1:] = np.cumsum(lens)[:-1]
        d_pcm = torch.from_numpy(pcm).cuda()
        d_out = torch.zeros(len(lens), fresh.dim, device="cuda")
        fresh.embed_device(d_pcm, offs, lens, d_out, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        got_dev = d_out.cpu().numpy()
        got_host = fresh.embed_batch(clips)
    finally:
        fresh.close()
    for i in range(len(clips)):
        assert _cos(got_dev[i], want[i]) >= 0.99999, i
        assert _cos(got_host[i], want[i]) >= 0.99999, i


def test_page_locked_clips_copied_directly(resnet):
    """Clips in page-locked host memory (voicedetect_b200_host_register) reach the device
    by DMA from the caller's buffer instead of the engine's gather. The embeddings must
    equal the pageable call's bit for bit, for f32 and int16 input, with every clip
    locked and with a batch that mixes locked and pageable clips (gathered). Clips
    stored in ascending length are copied one by one (the engine runs them longest
    first, so neighbours in its order are not neighbours in memory); stored in
    descending length they follow one another in both and go as merged copies."""
    for lens in ([16000 + 1000 * i for i in range(12)], [27000 - 1000 * i for i in range(12)]):
        _check_page_locked(resnet, lens)


def _check_page_locked(resnet, lens):
    import vd_b200
    _, model = resnet
    parts = [vd_synth.clip_f32(vd_synth.make_clip(700 + i, n)) for i, n in enumerate(lens)]
    pcm = np.concatenate(parts)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    clips = [pcm[o:o + n] for o, n in zip(offs, lens)]
    pcm16 = np.round(pcm * 32768.0).astype(np.int16)
    clips16 = [pcm16[o:o + n] for o, n in zip(offs, lens)]
    want = model.embed_batch(clips)
    want16 = model.embed_batch_s16(clips16)
    locked = []
    try:
        for a in (pcm, pcm16):
            assert vd_b200.host_register(a), vd_b200.last_error()
            locked.append(a)
        np.testing.assert_array_equal(model.embed_batch(clips), want)
        np.testing.assert_array_equal(model.embed_batch_s16(clips16), want16)
        mixed = [c if i % 2 else c.copy() for i, c in enumerate(clips)]  # copies are pageable
        np.testing.assert_array_equal(model.embed_batch(mixed), want)
    finally:
        for a in locked:
            vd_b200.host_unregister(a)


def test_verify_verdicts_match_oracle(resnet, tmp_path):
    import wave
    m, model = resnet

    def write(path, clip16):
        with wave.open(str(path), "wb") as w:
            w.setnchannels(1)
            w.setsampwidth(2)
            w.setframerate(16000)
            w.writeframes(clip16.tobytes())

    a16 = vd_synth.make_clip(5, 48000)
    b16 = vd_synth.make_clip(6, 40000)
    pa, pb = tmp_path / "a.wav", tmp_path / "b.wav"
    write(pa, a16)
    write(pb, b16)
    ea = _oracle_embed(m, vd_synth.clip_f32(a16))
    eb = _oracle_embed(m, vd_synth.clip_f32(b16))
    want = 1.0 - float(np.dot(ea.astype(np.float64), eb.astype(np.float64)))
    dist, _ = model.verify_paths(str(pa), str(pb), 0.25)
    assert abs(dist - want) <= 2e-3  # tests/test_verify.cpp distance gate
    for thr in (want - 0.01, want + 0.01):
        assert model.verify_paths(str(pa), str(pb), thr)[1] == (want <= thr)
    assert _cos(model.embed_path(str(pa)), ea) >= COS_TOL
    d_same, ok_same = model.verify_paths(str(pa), str(pa), 0.25)
    assert abs(d_same) < 1e-4 and ok_same


def test_resampled_input(resnet):
    m, model = resnet
    pcm8k = vd_synth.clip_f32(vd_synth.make_clip(8, 24000))
    got = model.embed_pcm(pcm8k, sample_rate=8000)
    want = _oracle_embed(m, oracle.resample_linear(pcm8k, 8000, 16000))
    assert _cos(got, want) >= COS_TOL


def test_error_paths(resnet):
    import vd_b200
    _, model = resnet
    with pytest.raises(vd_b200.VoiceDetectError, match="no frames"):
        model.embed_pcm(np.zeros(399, np.float32))
    with pytest.raises(vd_b200.VoiceDetectError, match="failed to load audio"):
        model.embed_path("/nonexistent.wav")
    assert model._L.voicedetect_capi_analyze_path_json(model.ctx, b"x.wav") is None
    assert "analyze" in model.last_error()
    # the context stays usable after errors
    pcm = vd_synth.clip_f32(vd_synth.make_clip(9, 16000))
    assert model.embed_pcm(pcm).shape == (256,)


@pytest.mark.parametrize("dtype", ["f16", "q8_0"])
def test_quantized_weights(tmp_path, cuda_lib, dtype):
    m = vd_synth.resnet34_model(4)
    path = tmp_path / f"m_{dtype}.gguf"
    vd_synth.write_resnet_gguf(str(path), m, dtype)
    mq = vd_synth.f16_model(m) if dtype == "f16" else vd_synth.quantize_q8_0_model(m)
    model = cuda_lib.Model(str(path))
    try:
        pcm = vd_synth.clip_f32(vd_synth.make_clip(10, 32000))
        assert _cos(model.embed_pcm(pcm), _oracle_embed(mq, pcm)) >= COS_TOL
    finally:
        model.close()


def test_device_path_matches_host_path(resnet):
    import torch
    m, model = resnet
    lens = [32000, 16000, 48000]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(400 + i, n)) for i, n in enumerate(lens)]
    host = model.embed_batch(clips)
    flat = torch.from_numpy(np.concatenate(clips)).cuda()
    offs = np.cumsum([0] + lens[:-1])
    out = torch.empty(len(clips), 256, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    model.embed_device(flat, offs, lens, out, s.cuda_stream)
    torch.cuda.synchronize()
    dev = out.cpu().numpy()
    assert np.allclose(dev, host, atol=1e-6)
    # metadata staging + fbank + cmn + stem + 32 convs + TSTP, FC, finish
    assert model.last_launches() == 39


def test_identify_matches_oracle(resnet):
    _, model = resnet
    rng = np.random.default_rng(3)
    reg = rng.standard_normal((1000, 256)).astype(np.float32)
    reg /= np.linalg.norm(reg, axis=1, keepdims=True)
    reg[500] = reg[17]  # an exact duplicate: the tie goes to the lower index
    q = reg[[17, 3, 999]] + 0.01 * rng.standard_normal((3, 256)).astype(np.float32)
    q = np.concatenate([q, rng.standard_normal((40, 256)).astype(np.float32)])
    idx, sc = model.identify(q, reg, k=5)
    widx, wsc = oracle.identify(q, reg, k=5)
    assert np.array_equal(idx, widx)
    assert np.allclose(sc, wsc, atol=1e-5)
    assert idx[0, 0] == 17 and idx[0, 1] == 500


@pytest.mark.parametrize("n_reg,dim,k", [(70001, 64, 5), (3000, 256, 64), (257, 48, 1)])
def test_identify_chunks_and_k(resnet, n_reg, dim, k):
    """Registries larger than one score chunk (32,768 rows for few queries), the
    largest k, k = 1, and sizes that are not multiples of the 128-row tiles, with
    duplicate rows that must tie-break to the lower index."""
    _, model = resnet
    rng = np.random.default_rng(n_reg)
    reg = rng.standard_normal((n_reg, dim)).astype(np.float32)
    reg /= np.linalg.norm(reg, axis=1, keepdims=True)
    reg[n_reg - 1] = reg[5]
    reg[40000 % n_reg] = reg[6]
    q = np.concatenate([reg[[5, 6]] + 0.001 * rng.standard_normal((2, dim)).astype(np.float32),
                        rng.standard_normal((37, dim)).astype(np.float32)])
    idx, sc = model.identify(q, reg, k=k)
    widx, wsc = oracle.identify(q, reg, k=k)
    assert np.array_equal(idx, widx)
    assert np.allclose(sc, wsc, atol=1e-5)


def test_repeated_shapes_replay_graphs(resnet):
    """A bucket shape seen again is replayed from a captured CUDA graph: results stay
    equal to the oracle, for new audio of the same lengths and for reordered clips
    (the per-clip metadata is refreshed in device memory before every replay)."""
    m, model = resnet
    lens = [32000, 24000, 16000 + 160 * 3]
    for rnd in range(4):
        clips = [vd_synth.clip_f32(vd_synth.make_clip(500 + 10 * rnd + i, n))
                 for i, n in enumerate(lens)]
        if rnd == 3:
            clips = clips[::-1]
        got = model.embed_batch(clips)
        for i, c in enumerate(clips):
            assert _cos(got[i], _oracle_embed(m, c)) >= COS_TOL, (rnd, i)
    # device path: same shapes four times
    import torch
    pcm = np.concatenate([vd_synth.clip_f32(vd_synth.make_clip(600 + i, n))
                          for i, n in enumerate(lens)])
    offs = np.cumsum([0] + lens[:-1]).astype(np.int64)
    d_pcm = torch.from_numpy(pcm).cuda()
    outs = []
    for _ in range(4):
        d_out = torch.zeros(len(lens), model.dim, device="cuda")
        model.embed_device(d_pcm, offs, lens, d_out)
        model.sync()
        outs.append(d_out.cpu().numpy())
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
