"""Pins the CPU oracle (oracle/vd_oracle.c) before anything is checked against it.

* against the reference's own kernels compiled from its sources
  (oracle/_ref/libvdref.so) on the shapes of the reference's model-free unit
  test tests/test_blocked.cpp, and on FBank / full ResNet forwards;
* against committed golden vectors (tests/golden/, made by make_golden.py):
  torchaudio Kaldi FBank, and outputs of the reference kernels.
Runs on CPU (no GPU needed).
"""
from pathlib import Path

import numpy as np
import pytest

import oracle
import vd_synth

GOLD = Path(__file__).resolve().parent / "golden"

# reference gates: conv max|d| <= 1e-4 (tests/test_blocked.cpp:107), FBank
# max|d| <= 1e-3 and cosine >= 0.9999 (tests/test_fbank.cpp:56-59)
CONV_TOL = 1e-4
FBANK_TOL = 1e-3


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0.0 and nb == 0.0:  # e.g. a one-frame clip: CMN zeroes everything
        return 1.0
    return float(a @ b / (na * nb))


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("reference kernels library not built")
    return oracle


def test_fbank_matches_torchaudio_golden():
    g = np.load(GOLD / "fbank_torchaudio.npz")
    for i in range(3):
        pcm = vd_synth.clip_f32(g[f"clip{i}"])
        want = g[f"fbank{i}"]
        got = oracle.fbank(pcm)
        assert got.shape == want.shape
        assert np.abs(got - want).max() <= FBANK_TOL
        assert _cos(got, want) >= 0.9999


def test_fbank_matches_reference_kernel(ref):
    for seed, n in ((1, 48000), (2, 16123), (3, 400), (4, 559)):
        pcm = vd_synth.clip_f32(vd_synth.make_clip(seed, n))
        a, b = oracle.fbank(pcm), ref.ref_fbank(pcm)
        assert a.shape == b.shape
        assert np.array_equal(a, b), np.abs(a - b).max()


def test_fbank_no_frames():
    pcm = np.zeros(399, np.float32)
    assert oracle.fbank(pcm).shape == (80, 0)


def test_conv_kat_golden():
    """C restatement vs the reference kernels' outputs on test_blocked shapes."""
    import importlib.util
    g = np.load(GOLD / "ref_conv_kat.npz")
    spec = importlib.util.spec_from_file_location("make_golden", GOLD / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    for i, (W, H, IC, OC, s, br, k) in enumerate(mg.CONV_KAT):
        x, w, b = mg.conv_inputs(i, W, H, IC, OC, k)
        y = oracle.conv2d(x, w, s, b if br else None, br)
        want = g[f"y{i}"]
        assert y.shape == want.shape
        assert np.abs(y - want).max() <= CONV_TOL


@pytest.mark.parametrize("stride", [1, 2])
def test_conv_matches_reference_kernel(ref, stride):
    rng = np.random.default_rng(9)
    for (W, H, IC, OC) in ((37, 13, 32, 32), (26, 10, 64, 64), (9, 7, 128, 256)):
        x = rng.uniform(-1, 1, (IC, H, W)).astype(np.float32)
        w = rng.uniform(-1, 1, (OC, IC, 3, 3)).astype(np.float32)
        b = rng.uniform(-1, 1, OC).astype(np.float32)
        assert np.array_equal(oracle.conv2d(x, w, stride, b, True),
                              ref.ref_conv3x3(x, w, stride, b, True))
        w1 = rng.uniform(-1, 1, (OC, IC, 1, 1)).astype(np.float32)
        assert np.array_equal(oracle.conv2d(x, w1, stride, b), ref.ref_conv1x1(x, w1, stride, b))
        if stride == 1:
            wi = ref.ref_winograd3x3(x, w)
            assert np.abs(wi - oracle.conv2d(x, w, 1)).max() <= CONV_TOL * max(1, np.abs(wi).max())


def test_resnet_tiny_golden():
    g = np.load(GOLD / "ref_resnet_tiny.npz")
    m = vd_synth.tiny_resnet_model(5, n_mels=80)
    feats = oracle.fbank(g["pcm"])
    emb, pre = oracle.resnet34_embed(m, feats)
    assert np.abs(pre - g["prenorm"]).max() <= 1e-3 * max(1.0, np.abs(g["prenorm"]).max())
    assert _cos(emb, g["emb"]) >= 0.999999


def test_resnet34_matches_reference_kernels(ref):
    m = vd_synth.resnet34_model(3)
    pcm = vd_synth.clip_f32(vd_synth.make_clip(77, 16000 + 160 * 13))
    feats = oracle.fbank(pcm)
    e0, p0 = oracle.resnet34_embed(m, feats)
    e1, p1 = ref.RefResNet34(m).embed(feats)
    assert np.array_equal(p0, p1)
    assert np.array_equal(e0, e1)


def test_eres2net_tiny_golden():
    g = np.load(GOLD / "ref_eres2net_tiny.npz")
    m = vd_synth.tiny_eres2net_model(6, n_mels=80)
    feats = oracle.fbank(g["pcm"])
    emb, pre = oracle.eres2net_embed(m, feats)
    assert pre.shape == (512,)
    assert np.abs(pre - g["prenorm"]).max() <= 1e-3 * max(1.0, np.abs(g["prenorm"]).max())
    assert _cos(emb, g["emb"]) >= 0.999999


def test_eres2net_matches_reference_kernels(ref):
    """Restated ERes2Net glue + C conv vs the same glue on the reference's blocked
    conv kernels: bit-identical (same accumulation order)."""
    m = vd_synth.tiny_eres2net_model(8, n_mels=80)
    pcm = vd_synth.clip_f32(vd_synth.make_clip(78, 16000 + 160 * 9))
    feats = oracle.fbank(pcm)
    e0, p0 = oracle.eres2net_embed(m, feats)
    e1, p1 = ref.RefERes2Net(m).embed(feats)
    assert np.array_equal(p0, p1)
    assert np.array_equal(e0, e1)


def test_eres2net_conv_manifest():
    """The full ERes2Net-base manifest has 96 convs, stem included, in forward-execution
    order (src/model_loader.hpp:68-80) and a 2*512*10 pooled vector at 80 mels."""
    m = vd_synth.eres2net_model(0)
    assert len(m["convs"]) == 96
    assert m["seg_w"].shape == (512, 2 * 512 * 10)
    assert sum(c["b"] is None for c in m["convs"]) == 3  # the cross-stage downsamples


def test_q8_0_roundtrip_matches_gguf_dequant(tmp_path):
    """The q8_0 model the oracle sees equals what a q8_0 GGUF carries."""
    gguf = pytest.importorskip("gguf")
    m = vd_synth.tiny_resnet_model(2, n_mels=16)
    q = vd_synth.quantize_q8_0_model(m)
    path = tmp_path / "q.gguf"
    vd_synth.write_resnet_gguf(str(path), m, "q8_0")
    r = gguf.GGUFReader(str(path))
    t = {x.name: x for x in r.tensors}
    w = t["blk1.conv1.weight"]
    assert w.tensor_type == gguf.GGMLQuantizationType.Q8_0
    deq = gguf.quants.dequantize(w.data, gguf.GGMLQuantizationType.Q8_0)
    oc, ic = q["blocks"][1]["conv1_w"].shape[:2]
    ohwi = deq.reshape(oc, 3, 3, ic)
    assert np.array_equal(ohwi.transpose(0, 3, 1, 2), q["blocks"][1]["conv1_w"])


def test_identify_oracle_ties():
    reg = np.eye(4, dtype=np.float32)
    reg = np.concatenate([reg, reg[:1]])  # row 4 duplicates row 0
    q = np.array([[1, 0, 0, 0]], np.float32)
    idx, sc = oracle.identify(q, reg, k=3)
    assert idx[0, 0] == 0 and idx[0, 1] == 4
    assert sc[0, 0] == pytest.approx(1.0) and sc[0, 1] == pytest.approx(1.0)


def test_resample_linear():
    x = np.arange(10, dtype=np.float32)
    y = oracle.resample_linear(x, 8000, 16000)
    assert len(y) == 20
    assert y[0] == 0 and y[1] == pytest.approx(0.5) and y[-1] == 9


def test_ecapa_tiny_golden():
    """numpy ECAPA oracle (oracle/ecapa.py) vs the committed golden made by an
    independent float64 torch formulation on torchaudio FBank features."""
    g = np.load(GOLD / "ref_ecapa_tiny.npz")
    m = vd_synth.tiny_ecapa_model(7, n_mels=80)
    for i in range(2):
        emb, pre = oracle.ecapa_embed(m, g[f"feats{i}"])
        want = g[f"prenorm{i}"]
        assert np.abs(pre - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
        assert _cos(emb, g[f"emb{i}"]) >= 0.999999
        # through the oracle's own FBank (pinned to torchaudio at 1e-3 above)
        emb2, _ = oracle.ecapa_embed(m, oracle.fbank(g[f"pcm{i}"]))
        assert _cos(emb2, g[f"emb{i}"]) >= 0.99999


def test_ecapa_reflect_index():
    """reflect_pad_time's index list (src/encoder.cpp:36-44): no edge repeat, and
    a clip must be longer than the padding."""
    from oracle.ecapa import reflect_index
    assert reflect_index(5, 4).tolist() == [4, 3, 2, 1, 0, 1, 2, 3, 4, 3, 2, 1, 0]
    assert reflect_index(7, 2).tolist() == [2, 1, 0, 1, 2, 3, 4, 5, 6, 5, 4]
    with pytest.raises(ValueError):
        reflect_index(4, 4)


def test_ecapa_gguf_layout(tmp_path):
    """write_ecapa_gguf follows the reference converter: verbatim names, KV dims,
    only the 1x1 MFA weight quantised and stored squeezed to 2-D."""
    gguf = pytest.importorskip("gguf")
    m = vd_synth.tiny_ecapa_model(2, n_mels=80)
    path = tmp_path / "e.gguf"
    vd_synth.write_ecapa_gguf(str(path), m, "f16")
    r = gguf.GGUFReader(str(path))
    t = {x.name: x for x in r.tensors}
    assert set(t) == set(m["sd"])
    assert t["mfa.conv.conv.weight"].tensor_type == gguf.GGMLQuantizationType.F16
    assert list(t["mfa.conv.conv.weight"].shape) == [3 * 64, 96]  # ne = [IC, OC]
    for name in ("fc.conv.weight", "asp.tdnn.conv.conv.weight", "blocks.1.tdnn1.conv.conv.weight",
                 "blocks.1.se_block.conv1.conv.weight", "blocks.0.conv.conv.weight"):
        assert t[name].tensor_type == gguf.GGMLQuantizationType.F32, name
    assert list(t["blocks.0.conv.conv.weight"].shape) == [5, 80, 64]  # ne = [K, IC, OC]
    kv = {f.name: f for f in r.fields.values()}
    assert "voicedetect.ecapa.res2net_scale" in kv


def test_ecapa_f16_weights_are_well_conditioned():
    """The calibrated synthetic ECAPA is not chaotic: rounding its conv weights to
    f16 moves the embedding far less than the 0.9999 gate."""
    m = vd_synth.tiny_ecapa_model(3, n_mels=80)
    feats = oracle.fbank(vd_synth.clip_f32(vd_synth.make_clip(31, 24000)))
    a, _ = oracle.ecapa_embed(m, feats)
    b, _ = oracle.ecapa_embed(vd_synth.f16_ecapa_model(m), feats)
    assert _cos(a, b) >= 0.99999


def test_campplus_tiny_golden():
    """numpy CAM++ oracle (oracle/campplus.py) vs the committed golden made by an
    independent float64 torch formulation on torchaudio FBank features (one clip
    spans two 100-frame context segments)."""
    g = np.load(GOLD / "ref_campplus_tiny.npz")
    m = vd_synth.tiny_campplus_model(9, n_mels=80)
    for i in range(2):
        emb, pre = oracle.campplus_embed(m, g[f"feats{i}"])
        want = g[f"prenorm{i}"]
        assert np.abs(pre - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
        assert _cos(emb, g[f"emb{i}"]) >= 0.999999
        emb2, _ = oracle.campplus_embed(m, oracle.fbank(g[f"pcm{i}"]))
        assert _cos(emb2, g[f"emb{i}"]) >= 0.99999


def test_campplus_manifest_and_gguf(tmp_path):
    """The full CAM++ manifest: 225 convs and 55 runtime BatchNorms in execution
    order (the converter's assertion, scripts/convert_voicedetect_to_gguf.py), written
    with the reference's voicedetect.campplus.* keys."""
    gguf = pytest.importorskip("gguf")
    m = vd_synth.campplus_model(0, calibrate=False)
    assert len(m["convs"]) == 225 and len(m["bns"]) == 55
    assert m["convs"][-1]["w"].shape == (192, 1024, 1)
    path = tmp_path / "c.gguf"
    vd_synth.write_campplus_gguf(str(path), m, "f16")
    r = gguf.GGUFReader(str(path))
    kv = {f.name for f in r.fields.values()}
    assert {"voicedetect.campplus.conv_weight", "voicedetect.campplus.bn_prefix",
            "voicedetect.campplus.emb_bn_mean"} <= kv


@pytest.mark.parametrize("T", [1, 3, 199, 201])
def test_campplus_oracle_edge_lengths(T):
    """CAM++ oracle vs the float64 torch formulation at the lengths where the forward
    changes shape: one TDNN frame (no std correction), exactly one 100-frame context
    segment, and one frame into a second segment."""
    m = vd_synth.tiny_campplus_model(9, n_mels=80)
    rng = np.random.default_rng(T)
    feats = (rng.standard_normal((80, T)) * 1.5).astype(np.float32)
    emb, pre = oracle.campplus_embed(m, feats)
    torch = pytest.importorskip("torch")
    temb, tpre = vd_synth.campplus_forward_torch(
        m, torch.from_numpy(feats[None].astype(np.float64)))
    assert np.abs(pre - tpre[0]).max() <= 1e-4 * max(1.0, np.abs(tpre[0]).max())
    assert _cos(emb, temb[0]) >= 0.999999
