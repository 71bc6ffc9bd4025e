"""End-to-end ERes2Net parity through the C ABI (voicedetect_capi_*): PCM ->
FBank -> CMN+stem -> the Res2Net body (clamp, split/concat, AFF, cross-stage
fusion; src/encoder_eres2net.cpp:36-226) on tcgen05 convs -> TSTP+FC+L2,
against the CPU oracle (oracle/vd_oracle.c vdo_eres2net_forward, pinned
bit-exact to the reference's own conv kernels in tests/test_oracle.py).

The GGUF carries f16 weights, so the oracle runs the same
f16-rounded weights widened to f32. Gate: embedding cosine >= 0.9999.
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


def _model(tmp_path_factory, cuda_lib, m, dtype, name):
    path = tmp_path_factory.mktemp("e") / name
    vd_synth.write_eres2net_gguf(str(path), m, dtype)
    return cuda_lib.Model(str(path))


@pytest.fixture(scope="module")
def eres_f16(tmp_path_factory, cuda_lib):
    m = vd_synth.eres2net_model(0)
    model = _model(tmp_path_factory, cuda_lib, m, "f16", "eres2net_f16.gguf")
    yield vd_synth.quantize_model_f16(m), model
    model.close()


def _oracle(m, pcm):
    return oracle.eres2net_embed(m, oracle.fbank(pcm))[0]


def test_eres2net_embed_matches_oracle(eres_f16):
    m, model = eres_f16
    pcm = vd_synth.clip_f32(vd_synth.make_clip(2, 48000))
    got = model.embed_pcm(pcm)
    assert got.shape == (512,)
    assert abs(float(np.linalg.norm(got)) - 1.0) < 1e-3
    assert _cos(got, _oracle(m, pcm)) >= COS_TOL


def test_eres2net_config2_clip(eres_f16):
    """A 10 s clip (998 frames), the clip length of the ERes2Net benchmark config."""
    m, model = eres_f16
    pcm = vd_synth.clip_f32(vd_synth.make_clip(3, 160000))
    assert _cos(model.embed_pcm(pcm), _oracle(m, pcm)) >= COS_TOL


def test_eres2net_ragged_batch(eres_f16):
    m, model = eres_f16
    lens = [32000, 16000, 401 + 160 * 5, 40000, 20000 + 77]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(200 + i, n)) for i, n in enumerate(lens)]
    got = model.embed_batch(clips)
    for i, c in enumerate(clips):
        assert _cos(got[i], _oracle(m, c)) >= COS_TOL, i
    assert _cos(model.embed_pcm(clips[2]), got[2]) >= 0.99999


def test_eres2net_tiny_f32(tmp_path_factory, cuda_lib):
    """A different topology (blocks 1/1/2/1) from an f32 GGUF: the plan follows the
    manifest, not a fixed layer count."""
    m = vd_synth.tiny_eres2net_model(6, n_mels=80)
    model = _model(tmp_path_factory, cuda_lib, m, "f32", "eres2net_tiny.gguf")
    try:
        g = np.load(__import__("pathlib").Path(__file__).parent / "golden" /
                    "ref_eres2net_tiny.npz")
        got = model.embed_pcm(g["pcm"])
        # the committed reference-kernel output for this model and clip
        assert _cos(got, g["emb"]) >= COS_TOL
    finally:
        model.close()


def test_eres2net_random_bn_statistics(tmp_path_factory, cuda_lib):
    """With the random BatchNorm statistics of the ResNet config (mean N(0, 0.1), var
    U(0.5, 1.5), unrelated to the activations) the 96-conv ERes2Net is chaotic: a CPU
    float32 forward whose stored activations are rounded to f16 (and nothing else
    changed) reaches only cosine ~0.9994 against the float32 oracle on this clip. The
    GPU path stores f16 activations, so it is held to that bound here, not to 0.9999."""
    m = vd_synth.eres2net_model(0, calibrate=False)
    model = _model(tmp_path_factory, cuda_lib, m, "f16", "eres2net_rand_bn.gguf")
    try:
        pcm = vd_synth.clip_f32(vd_synth.make_clip(2, 48000))
        got = model.embed_pcm(pcm)
        assert _cos(got, _oracle(vd_synth.quantize_model_f16(m), pcm)) >= 0.999
    finally:
        model.close()
