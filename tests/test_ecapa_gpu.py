"""ECAPA-TDNN on the B200 engine.

Op level: vdb_conv1d (the tensor-core TDNN conv, src/encoder.cpp:65-167) against
torch float32 conv1d with SpeechBrain's reflect padding at each clip's own length,
on ragged batches: kernel 1/3/5, dilations, the ReLU -> BatchNorm (-> tanh)
epilogues, a per-clip bias, two input segments, the reflection rows it writes,
the y + addend second output and the f32 output. Gate: rel-L2 <= 1e-3.

End to end through the C ABI: PCM -> FBank -> CMN -> stem -> SE-Res2Net blocks
-> MFA -> attentive statistics pooling -> fc -> L2 against the numpy oracle
(oracle/ecapa.py) on the weights the GGUF carries. Gate: cosine >= 0.9999 and
identical verify verdicts.
"""
import numpy as np
import pytest

import oracle
import vd_synth

pytestmark = pytest.mark.gpu

COS_TOL = 0.9999
REL_TOL = 1e-3


def _cos(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def _ref_conv(torch, x, w, b, tv, dil):
    """Per clip: reflect-pad the valid frames, conv1d (f32). x (B, IC, T) -> list."""
    import torch.nn.functional as Fn
    out = []
    k = w.shape[-1]
    pad = (k - 1) // 2 * dil
    for i, t in enumerate(tv):
        xb = x[i:i + 1, :, :t]
        if pad:
            xb = Fn.pad(xb, (pad, pad), mode="reflect")
        out.append(Fn.conv1d(xb, w, b, dilation=dil)[0])
    return out


# (B, T, pad, ic, oc, k, dil, act, two_seg, clip_bias, ysum, y_f32, tile_m, tile_n)
CASES = {
    "stem_k5": (3, 61, 4, 80, 128, 5, 1, 3, False, False, False, False, 0, 0),
    "tdnn_1x1": (4, 70, 4, 256, 256, 1, 1, 3, False, False, False, False, 0, 0),
    "group_k3_d2": (3, 50, 4, 64, 64, 3, 2, 3, False, False, True, False, 0, 0),
    "group_k3_d4": (3, 50, 4, 128, 128, 3, 4, 3, False, False, True, False, 128, 0),
    "tdnn2_two_seg": (2, 40, 4, 32, 256, 1, 1, 3, True, False, False, False, 0, 128),
    "asp_tdnn_tanh": (3, 45, 4, 192, 64, 1, 1, 4, False, True, False, False, 0, 0),
    "asp_conv_f32": (3, 45, 4, 64, 192, 1, 1, 0, False, False, False, True, 0, 0),
    "wide_1536": (2, 33, 4, 128, 1536, 1, 1, 3, False, False, False, False, 256, 256),
}


@pytest.mark.parametrize("pair", [1, 0], ids=["pair", "single"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_conv1d_matches_torch(cuda_lib, name, pair):
    """pair 1: two-SM cta_group::2 tiles (where the tiling allows them), 0: one CTA
    per tile, multi-tap convs fed by one input halo per channel block."""
    import torch
    B, T, pad, ic, oc, k, dil, act, two_seg, use_cb, use_sum, y_f32, tm, tn = CASES[name]
    if pair and tm not in (0, 256):
        pytest.skip("a CTA pair computes 256-row tiles")
    vd = cuda_lib
    g = torch.Generator().manual_seed(hash(name) % 1000)
    tv = [T] + [max(pad + 1, T - 7 * i - 3) for i in range(1, B)]
    x = torch.relu(torch.randn(B, ic, T, generator=g)).half().float()
    w = (torch.randn(oc, ic, k, generator=g) * (2.0 / (ic * k)) ** 0.5).half().float()
    b = torch.randn(oc, generator=g) * 0.1
    ic1 = 96 if two_seg else 0
    x1 = torch.relu(torch.randn(B, ic1, T, generator=g)).half().float() if two_seg else None
    w1 = (torch.randn(oc, ic1, 1, generator=g) * (2.0 / max(ic1, 1)) ** 0.5).half().float() \
        if two_seg else None
    sc = torch.rand(oc, generator=g) + 0.5
    sh = torch.randn(oc, generator=g) * 0.1
    cb = torch.randn(B, oc, generator=g) * 0.2 if use_cb else None
    add = torch.relu(torch.randn(B, oc, T, generator=g)).half().float() if use_sum else None

    ref = _ref_conv(torch, x, w, b, tv, dil)
    if two_seg:
        r1 = _ref_conv(torch, x1, w1, None, tv, 1)
        ref = [r + q for r, q in zip(ref, r1)]
    outs = []
    for i, r in enumerate(ref):
        if cb is not None:
            r = r + cb[i][:, None]
        if act in (3, 4):
            r = torch.relu(r) * sc[:, None] + sh[:, None]
            if act == 4:
                r = torch.tanh(r)
        outs.append(r)

    dev = torch.device("cuda")
    xs = vd.to_seq(x, pad, tv).to(dev)
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    kw = {}
    if two_seg:
        kw.update(x1=vd.to_seq(x1, pad, tv).to(dev), w1=w1[:, :, 0].half().contiguous().to(dev))
    if act in (3, 4):
        kw.update(bn_scale=sc.to(dev), bn_shift=sh.to(dev))
    if cb is not None:
        kw.update(clip_bias=cb.contiguous().to(dev))
    rows = vd.lib().vdb_seq_rows(B, T, pad)
    ysum = None
    if use_sum:
        ysum = torch.zeros(rows, oc, dtype=torch.float16, device=dev)
        kw.update(ysum=ysum, addend=vd.to_seq(add, pad, tv).to(dev))
    y = torch.zeros(rows, oc, dtype=torch.float32 if y_f32 else torch.float16, device=dev)
    # pair 0 on a multi-tap single-segment conv also exercises the 1-D halo feed
    halo = 1 if (not pair and k > 1 and not two_seg and tn == 0
                 and k * ic * oc * 2 <= 96 * 1024) else 0
    vd.conv1d(xs, vd.pack_conv1d_weight(w).to(dev), b.to(dev), tvd, batch=B, t=T, pad=pad,
              oc=oc, k0=k, dil0=dil, act=act, y=y, y_f32=y_f32, reflect=not y_f32,
              tile_m=tm, tile_n=tn, pair=pair, halo=halo, **kw)
    torch.cuda.synchronize()
    ys = y.float().cpu().reshape(B, T + 2 * pad, oc)
    for i, t in enumerate(tv):
        got = ys[i, pad:pad + t].t()
        assert _rel(got.numpy(), outs[i].numpy()) <= REL_TOL, (name, i)
        if not y_f32:
            # the reflection rows the kernel wrote mirror the stored frames exactly
            for j in range(1, pad + 1):
                assert torch.equal(ys[i, pad - j], ys[i, pad + j]), (name, i, j)
                assert torch.equal(ys[i, pad + t - 1 + j], ys[i, pad + t - 1 - j]), (name, i, j)
    if use_sum:
        ss = ysum.float().cpu().reshape(B, T + 2 * pad, oc)
        for i, t in enumerate(tv):
            want = (ys[i, pad:pad + t] + add[i, :, :t].t()).half().float()
            assert torch.equal(ss[i, pad:pad + t], want), (name, i)
            for j in range(1, pad + 1):
                assert torch.equal(ss[i, pad - j], ss[i, pad + j])


def test_conv1d_pair_rejects_odd_tiles(cuda_lib):
    import torch
    vd = cuda_lib
    dev = torch.device("cuda")
    B, T, pad = 1, 20, 1
    xs = torch.zeros(vd.lib().vdb_seq_rows(B, T, pad), 32, dtype=torch.float16, device=dev)
    w = torch.zeros(48, 1, 32, dtype=torch.float16, device=dev)
    tvd = torch.tensor([T], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="pair"):
        vd.conv1d(xs, w, None, tvd, batch=B, t=T, pad=pad, oc=48, pair=1)


def test_conv1d_rejects_reach_beyond_pad(cuda_lib):
    import torch
    vd = cuda_lib
    dev = torch.device("cuda")
    B, T, pad = 1, 20, 2
    xs = torch.zeros(vd.lib().vdb_seq_rows(B, T, pad), 32, dtype=torch.float16, device=dev)
    w = torch.zeros(32, 3, 32, dtype=torch.float16, device=dev)
    tvd = torch.tensor([T], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="pad"):
        vd.conv1d(xs, w, None, tvd, batch=B, t=T, pad=pad, oc=32, k0=3, dil0=3)


# ---------------------------------------------------------------------------
# end to end
# ---------------------------------------------------------------------------
def _model(tmp_path_factory, cuda_lib, m, dtype, name):
    path = tmp_path_factory.mktemp("ec") / name
    vd_synth.write_ecapa_gguf(str(path), m, dtype)
    return cuda_lib.Model(str(path))


@pytest.fixture(scope="module")
def ecapa_f16(tmp_path_factory, cuda_lib):
    """The BASELINE config-3 network (C 1024, scale 8, MFA 1536, 192-d), f16 GGUF."""
    m = vd_synth.ecapa_model(0)
    model = _model(tmp_path_factory, cuda_lib, m, "f16", "ecapa_f16.gguf")
    yield vd_synth.quantized_ecapa_model(m, "f16"), model
    model.close()


def _oracle(m, pcm):
    return oracle.ecapa_embed(m, oracle.fbank(pcm))[0]


def test_ecapa_embed_matches_oracle(ecapa_f16):
    m, model = ecapa_f16
    pcm = vd_synth.clip_f32(vd_synth.make_clip(5, 64000))  # 4 s, config 3
    got = model.embed_pcm(pcm)
    assert got.shape == (192,)
    assert abs(float(np.linalg.norm(got)) - 1.0) < 1e-3
    assert _cos(got, _oracle(m, pcm)) >= COS_TOL


def test_ecapa_ragged_batch(ecapa_f16):
    m, model = ecapa_f16
    lens = [64000, 16000, 400 + 160 * 4, 48000 + 333, 20000, 160000]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(300 + i, n)) for i, n in enumerate(lens)]
    got = model.embed_batch(clips)
    for i, c in enumerate(clips):
        assert _cos(got[i], _oracle(m, c)) >= COS_TOL, i
    # a clip alone and inside a bucket give the same embedding
    assert _cos(model.embed_pcm(clips[2]), got[2]) >= 0.99999


def test_ecapa_verdicts_match_oracle(ecapa_f16):
    """verify_paths semantics (src/model.cpp:65-78): distance = 1 - a.b, verdicts
    at the config threshold equal the oracle's."""
    m, model = ecapa_f16
    clips = [vd_synth.clip_f32(vd_synth.make_clip(400 + i, 32000 + 1000 * i)) for i in range(6)]
    got = model.embed_batch(clips)
    want = np.stack([_oracle(m, c) for c in clips])
    dg = 1.0 - got @ got.T
    dw = 1.0 - want @ want.T
    thr = float(np.median(dw[np.triu_indices(6, 1)]))
    assert np.array_equal(dg <= thr, dw <= thr) or np.abs(dg - dw).max() < 1e-3


def test_ecapa_replay_is_deterministic(ecapa_f16):
    """The third call of a bucket shape replays a CUDA graph: same bits as the first."""
    _, model = ecapa_f16
    clips = [vd_synth.clip_f32(vd_synth.make_clip(500 + i, 40000 + 160 * i)) for i in range(5)]
    a = model.embed_batch(clips)
    model.embed_batch(clips)
    c = model.embed_batch(clips)
    assert np.array_equal(a, c)


def test_ecapa_short_clip_is_refused(ecapa_f16):
    _, model = ecapa_f16
    pcm = vd_synth.clip_f32(vd_synth.make_clip(6, 400 + 160 * 3))  # 4 frames < pad + 1
    with pytest.raises(Exception, match="frames"):
        model.embed_pcm(pcm)


def test_ecapa_tiny_golden(tmp_path_factory, cuda_lib):
    """The narrow f32 model of the committed golden (torch float64 forward)."""
    m = vd_synth.tiny_ecapa_model(7, n_mels=80)
    model = _model(tmp_path_factory, cuda_lib, m, "f32", "ecapa_tiny.gguf")
    try:
        g = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "ref_ecapa_tiny.npz")
        got = model.embed_batch([g["pcm0"], g["pcm1"]])
        for i in range(2):
            assert _cos(got[i], g[f"emb{i}"]) >= COS_TOL, i
    finally:
        model.close()


def test_ecapa_q8_0_mfa(tmp_path_factory, cuda_lib):
    """q8_0 GGUF: only the MFA weight is quantised (the reference converter's plan)."""
    m = vd_synth.tiny_ecapa_model(9, n_mels=80)
    model = _model(tmp_path_factory, cuda_lib, m, "q8_0", "ecapa_q8.gguf")
    try:
        mq = vd_synth.quantized_ecapa_model(m, "q8_0")
        pcm = vd_synth.clip_f32(vd_synth.make_clip(8, 30000))
        assert _cos(model.embed_pcm(pcm), _oracle(mq, pcm)) >= COS_TOL
    finally:
        model.close()


def test_ecapa_profile_counts_convs(ecapa_f16):
    """Profiling brackets every tensor-core conv of a bucket (stem, 3 x (tdnn1 + 7
    Res2Net convs + tdnn2), MFA, the two attention convs) and leaves no error behind."""
    _, model = ecapa_f16
    clips = [vd_synth.clip_f32(vd_synth.make_clip(600 + i, 64000)) for i in range(4)]
    model.profile(True)
    model.profile_read()
    model.embed_batch(clips)
    ms, flops, n = model.profile_read()
    stages = model.profile_stages()
    model.profile(False)
    assert n == 31 and ms > 0 and flops > 0
    assert stages["conv"] > 0 and stages["pool"] > 0
    assert model.embed_batch(clips).shape == (4, 192)
