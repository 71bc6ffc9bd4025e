"""CAM++ on the B200 engine.

Op level (vdb_conv / vdb_conv1d extensions the CAM++ forward uses) against torch
float32 convs on ragged batches, gate rel-L2 <= 1e-3:
  * 2-D conv with a frequency-only stride 2 (stride code 3) reading the FPHASE layout,
    with the fused 1x1 shortcut as a second segment and an FPHASE output (y_phase 2);
  * the FCM's last conv writing the TDNN's time-phase input (y_phase 3);
  * the TDNN conv with time stride 2 over that input, zero-padded output (reflect 2);
  * the CAM layer's dilated conv with the per-segment gate in its epilogue (act 5);
  * the dense layers' 1x1 convs with the BatchNorm + ReLU of their input applied to
    the A tiles in shared memory (the input prologue).

End to end through the C ABI: PCM -> FBank -> CMN -> FCM -> TDNN -> dense blocks
-> statistics pooling -> dense head -> L2 against the numpy oracle
(oracle/campplus.py, pinned to a float64 torch formulation) on the weights the
GGUF carries. Gate: cosine >= 0.9999 and identical verify verdicts.
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


def _mask_t(x, tv):
    """Zero frames t >= tv[b] of a (B, ..., T) tensor."""
    x = x.clone()
    for b, t in enumerate(tv):
        x[b, ..., t:] = 0
    return x


@pytest.mark.parametrize("halo,tile_m", [(0, 0), (-1, 0), (1, 512)],
                         ids=["auto", "tap", "halo512"])
@pytest.mark.parametrize("F,T", [(80, 37), (41, 29)])
def test_conv2d_freq_stride(cuda_lib, F, T, halo, tile_m):
    """Block 0 of an FCM stage: conv1 3x3 stride (2, 1) from FPHASE (fed per tap, or
    by one halo per frequency plane with the weights resident); conv2 3x3 + the 1x1
    stride-(2, 1) shortcut (second K segment) -> ReLU, stored as FPHASE."""
    import torch
    import torch.nn.functional as Fn
    vd = cuda_lib
    g = torch.Generator().manual_seed(F * 100 + T)
    B, C = 3, 32
    tv = [T, T - 5, 9]
    Fo = vd.out_extent(F, 2)
    x = _mask_t(torch.relu(torch.randn(B, C, F, T, generator=g)).half().float(), tv)
    w1 = (torch.randn(C, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).half().float()
    w2 = (torch.randn(C, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).half().float()
    ws = (torch.randn(C, C, 1, 1, generator=g) * (2.0 / C) ** 0.5).half().float()
    b1 = torch.randn(C, generator=g) * 0.1
    b2 = torch.randn(C, generator=g) * 0.1
    r1 = _mask_t(torch.relu(Fn.conv2d(x, w1, b1, stride=(2, 1), padding=1)), tv)
    r1h = r1.half().float()
    r2 = _mask_t(torch.relu(Fn.conv2d(r1h, w2, b2, padding=1) + Fn.conv2d(x, ws, None,
                                                                          stride=(2, 1))), tv)
    dev = torch.device("cuda")
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    xf = vd.to_fphase(x, tv).to(dev)
    y1 = vd.conv(xf, vd.pack_conv_weight(w1).to(dev), b1.to(dev), tvd, batch=B, t_out=T,
                 f_out=Fo, oc=C, k0=3, stride0=3, relu=True, halo=halo, tile_m=tile_m)
    got1 = vd.from_grid(y1, B, C, Fo, T).cpu()
    assert _rel(got1, r1) <= REL_TOL
    y2 = vd.conv(y1, vd.pack_conv_weight(w2).to(dev), b2.to(dev), tvd, batch=B, t_out=T,
                 f_out=Fo, oc=C, k0=3, x1=xf, w1=ws[:, :, 0, 0].half().contiguous().to(dev),
                 stride1=3, relu=True, y_phase=2)
    got2 = vd.from_fphase(y2, B, C, Fo, T).cpu()
    assert _rel(got2, r2) <= REL_TOL
    # the FPHASE output feeds the next stage's stride-(2, 1) conv
    Fq = vd.out_extent(Fo, 2)
    y3 = vd.conv(y2, vd.pack_conv_weight(w1).to(dev), b1.to(dev), tvd, batch=B, t_out=T,
                 f_out=Fq, oc=C, k0=3, stride0=3, relu=True, halo=halo, tile_m=tile_m)
    r3 = _mask_t(torch.relu(Fn.conv2d(vd.from_fphase(y2, B, C, Fo, T).cpu(), w1, b1,
                                      stride=(2, 1), padding=1)), tv)
    assert _rel(vd.from_grid(y3, B, C, Fq, T).cpu(), r3) <= REL_TOL


def test_fcm_to_tdnn_time_phase(cuda_lib):
    """FCM conv2 (3x3 stride (2, 1)) writes the TDNN's TPHASE input (channel f*C + c);
    the TDNN (k=5, stride 2, pad 2, ReLU) reads it and writes a zero-padded sequence."""
    import torch
    import torch.nn.functional as Fn
    vd = cuda_lib
    g = torch.Generator().manual_seed(11)
    B, C, F, T, P = 3, 32, 20, 41, 2
    tv = [T, 30, 7]
    Fo = vd.out_extent(F, 2)
    To = vd.out_extent(T, 2)
    x = _mask_t(torch.relu(torch.randn(B, C, F, T, generator=g)).half().float(), tv)
    w = (torch.randn(C, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).half().float()
    b = torch.randn(C, generator=g) * 0.1
    r = _mask_t(torch.relu(Fn.conv2d(x, w, b, stride=(2, 1), padding=1)), tv)  # (B, C, Fo, T)
    dev = torch.device("cuda")
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    ts = vd.conv(vd.to_fphase(x, tv).to(dev), vd.pack_conv_weight(w).to(dev), b.to(dev), tvd,
                 batch=B, t_out=T, f_out=Fo, oc=C, k0=3, stride0=3, relu=True, y_phase=3,
                 y_pad=P)
    # channel f*C + c of the sequence row
    want = r.permute(0, 2, 1, 3).reshape(B, Fo * C, T)
    got = vd.from_tphase(ts, B, Fo * C, T, P).cpu()
    assert _rel(got, want) <= REL_TOL
    # TDNN over the TPHASE input, written zero-padded into a wider buffer's slice
    oc = 64
    wt = (torch.randn(oc, Fo * C, 5, generator=g) * (2.0 / (5 * Fo * C)) ** 0.5).half().float()
    bt = torch.randn(oc, generator=g) * 0.1
    tq = [vd.out_extent(t, 2) for t in tv]
    tqd = torch.tensor(tq, dtype=torch.int32, device=dev)
    rows = vd.lib().vdb_seq_rows(B, To, P)
    wide = torch.full((rows, oc + 32), 7.0, dtype=torch.float16, device=dev)
    vd.conv1d(ts, vd.pack_conv1d_weight(wt).to(dev), bt.to(dev), tqd, batch=B, t=To, pad=P,
              oc=oc, k0=5, relu=True, y=wide[:, :oc], reflect=2, stride0=2)
    torch.cuda.synchronize()
    ys = wide.float().cpu().reshape(B, To + 2 * P, oc + 32)
    rh = got.half().float()
    for i, t in enumerate(tv):
        ref = torch.relu(Fn.conv1d(rh[i:i + 1, :, :t], wt, bt, stride=2, padding=2))[0]
        assert ref.shape[1] == tq[i]
        assert _rel(ys[i, P:P + tq[i], :oc].t(), ref) <= REL_TOL, i
        # zero padding: every other row of the slot is 0; the slice beyond oc untouched
        assert torch.count_nonzero(ys[i, :P, :oc]) == 0
        assert torch.count_nonzero(ys[i, P + tq[i]:, :oc]) == 0
        assert torch.all(ys[i, :, oc:] == 7.0)


@pytest.mark.parametrize("halo", [0, -1], ids=["halo", "tap"])
@pytest.mark.parametrize("dil", [1, 2])
def test_cam_gate_conv(cuda_lib, dil, halo):
    """CAM layer: linear_local (k=3, dilation, no bias, zero padding) times the
    per-(clip, segment) gate, stored zero-padded into a channel slice; fed by one
    input halo per channel block (the automatic choice) or one tile per tap."""
    import torch
    import torch.nn.functional as Fn
    vd = cuda_lib
    g = torch.Generator().manual_seed(20 + dil)
    B, T, P, ic, oc, seg = 4, 40, 2, 128, 32, 7
    tv = [T, 33, 8, 1]
    nseg = (T + seg - 1) // seg
    x = _mask_t(torch.relu(torch.randn(B, ic, T, generator=g)).half().float(), tv)
    w = (torch.randn(oc, ic, 3, generator=g) * (2.0 / (3 * ic)) ** 0.5).half().float()
    gate = torch.rand(B, nseg, oc, generator=g)
    dev = torch.device("cuda")
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    xs = vd.to_seq(x, P, tv, reflect=False).to(dev)
    rows = vd.lib().vdb_seq_rows(B, T, P)
    h = torch.full((rows, 96 + oc), 3.0, dtype=torch.float16, device=dev)
    vd.conv1d(xs, vd.pack_conv1d_weight(w).to(dev), None, tvd, batch=B, t=T, pad=P, oc=oc,
              k0=3, dil0=dil, act=5, gate=gate.to(dev), gate_seg=seg, gate_nseg=nseg,
              y=h[:, 96:], reflect=2, halo=halo)
    torch.cuda.synchronize()
    ys = h.float().cpu().reshape(B, T + 2 * P, 96 + oc)
    for i, t in enumerate(tv):
        r = Fn.conv1d(x[i:i + 1, :, :t], w, None, padding=dil, dilation=dil)[0]
        r = r * gate[i, torch.arange(t) // seg].t()
        assert _rel(ys[i, P:P + t, 96:].t(), r) <= REL_TOL, i
        assert torch.count_nonzero(ys[i, P + t:, 96:]) == 0
        assert torch.count_nonzero(ys[i, :P, 96:]) == 0
        assert torch.all(ys[i, :, :96] == 3.0)


@pytest.mark.parametrize("ic,ld", [(192, 256), (160, 160), (48, 64), (992, 1024)])
def test_conv1x1_bn_relu_prologue(cuda_lib, ic, ld):
    """Dense-layer 1x1 conv reading the first `ic` channels of a wider feature tensor
    with BN + ReLU applied to its A tiles in shared memory (64 / 32 / 16-channel K
    blocks, i.e. every TMA swizzle width). The prologue rounds scale and shift to f16
    and computes one f16 fused multiply-add with ReLU; the reference here is f32."""
    import torch
    import torch.nn.functional as Fn
    vd = cuda_lib
    g = torch.Generator().manual_seed(ic)
    B, T, P, oc = 3, 70, 2, 128
    tv = [T, 51, 3]
    x = _mask_t(torch.randn(B, ld, T, generator=g), tv).half().float()
    sc = torch.rand(ic, generator=g) + 0.5
    sh = torch.randn(ic, generator=g) * 0.3
    w = (torch.randn(oc, ic, 1, generator=g) * (2.0 / ic) ** 0.5).half().float()
    b = torch.randn(oc, generator=g) * 0.1
    a = torch.relu(x[:, :ic] * sc[None, :, None] + sh[None, :, None])
    dev = torch.device("cuda")
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    xs = vd.to_seq(x, P, tv, reflect=False).to(dev)
    y = vd.conv1d(xs[:, :ic], vd.pack_conv1d_weight(w).to(dev), b.to(dev), tvd, batch=B, t=T,
                  pad=P, oc=oc, relu=True, reflect=2, x_scale=sc.to(dev), x_shift=sh.to(dev))
    torch.cuda.synchronize()
    ys = y.float().cpu().reshape(B, T + 2 * P, oc)
    for i, t in enumerate(tv):
        r = torch.relu(Fn.conv1d(a[i:i + 1, :, :t], w, b))[0]
        assert _rel(ys[i, P:P + t].t(), r) <= REL_TOL, i
        assert torch.count_nonzero(ys[i, P + t:]) == 0


def test_conv1d_gate_needs_segments(cuda_lib):
    import torch
    vd = cuda_lib
    dev = torch.device("cuda")
    B, T, P = 1, 20, 1
    xs = torch.zeros(vd.lib().vdb_seq_rows(B, T, P), 32, dtype=torch.float16, device=dev)
    w = torch.zeros(32, 1, 32, dtype=torch.float16, device=dev)
    gate = torch.zeros(B, 1, 32, device=dev)
    tvd = torch.tensor([T], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="gate"):
        vd.conv1d(xs, w, None, tvd, batch=B, t=T, pad=P, oc=32, act=5, gate=gate, gate_seg=10,
                  gate_nseg=1)


# ---------------------------------------------------------------------------
# end to end
# ---------------------------------------------------------------------------
def _model(tmp_path_factory, cuda_lib, m, dtype, name):
    path = tmp_path_factory.mktemp("cp") / name
    vd_synth.write_campplus_gguf(str(path), m, dtype)
    return cuda_lib.Model(str(path))


def _oracle(m, pcm):
    return oracle.campplus_embed(m, oracle.fbank(pcm))[0]


@pytest.fixture(scope="module")
def campplus_f16(tmp_path_factory, cuda_lib):
    """The reference topology (FCM 32 channels, dense blocks 12 / 24 / 16, growth 32,
    512-channel output, 192-d), f16 GGUF."""
    m = vd_synth.campplus_model(0)
    model = _model(tmp_path_factory, cuda_lib, m, "f16", "campplus_f16.gguf")
    yield vd_synth.f16_campplus_model(m), model
    model.close()


def test_campplus_embed_matches_oracle(campplus_f16):
    m, model = campplus_f16
    pcm = vd_synth.clip_f32(vd_synth.make_clip(5, 64000))  # 4 s: two context segments
    got = model.embed_pcm(pcm)
    assert got.shape == (192,)
    assert abs(float(np.linalg.norm(got)) - 1.0) < 1e-3
    assert _cos(got, _oracle(m, pcm)) >= COS_TOL


def test_campplus_ragged_batch(campplus_f16):
    m, model = campplus_f16
    lens = [64000, 16000, 400 + 160 * 4, 48000 + 333, 20000, 112000]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(300 + i, n)) for i, n in enumerate(lens)]
    got = model.embed_batch(clips)
    for i, c in enumerate(clips):
        assert _cos(got[i], _oracle(m, c)) >= COS_TOL, i
    # a clip alone and inside a bucket give the same embedding
    assert _cos(model.embed_pcm(clips[2]), got[2]) >= 0.99999


def test_campplus_verdicts_match_oracle(campplus_f16):
    m, model = campplus_f16
    clips = [vd_synth.clip_f32(vd_synth.make_clip(400 + i, 32000 + 1000 * i)) for i in range(6)]
    got = model.embed_batch(clips)
    want = np.stack([_oracle(m, c) for c in clips])
    dg = 1.0 - got @ got.T
    dw = 1.0 - want @ want.T
    thr = float(np.median(dw[np.triu_indices(6, 1)]))
    assert np.array_equal(dg <= thr, dw <= thr) or np.abs(dg - dw).max() < 1e-3


def test_campplus_replay_is_deterministic(campplus_f16):
    """The third call of a bucket shape replays a CUDA graph: same bits as the first."""
    _, model = campplus_f16
    clips = [vd_synth.clip_f32(vd_synth.make_clip(500 + i, 40000 + 160 * i)) for i in range(5)]
    a = model.embed_batch(clips)
    model.embed_batch(clips)
    c = model.embed_batch(clips)
    assert np.array_equal(a, c)


def test_campplus_small_model_f32(tmp_path_factory, cuda_lib):
    """A narrow f32 model (FCM 16 channels, growth 32, two layers per block)."""
    m = vd_synth.campplus_model(4, m_channels=16, init_channels=64, growth=32, bn_size=2,
                                layers=(2, 2, 2), emb_dim=48)
    model = _model(tmp_path_factory, cuda_lib, m, "f32", "campplus_small.gguf")
    try:
        clips = [vd_synth.clip_f32(vd_synth.make_clip(700 + i, n))
                 for i, n in enumerate([36000, 9000, 560])]
        got = model.embed_batch(clips)
        for i, c in enumerate(clips):
            assert _cos(got[i], _oracle(m, c)) >= COS_TOL, i
    finally:
        model.close()


def test_campplus_q8_0(tmp_path_factory, cuda_lib):
    """q8_0 GGUF: the 1x1 Conv1d weights quantised (squeezed to [OC, IC], the
    converter's rule for rank <= 3 weights), dequantised at load."""
    m = vd_synth.campplus_model(5, m_channels=16, init_channels=64, growth=32, bn_size=2,
                                layers=(2, 2, 2), emb_dim=48)
    model = _model(tmp_path_factory, cuda_lib, m, "q8_0", "campplus_q8.gguf")
    try:
        mq = vd_synth.q8_campplus_model(m)
        clips = [vd_synth.clip_f32(vd_synth.make_clip(800 + i, n))
                 for i, n in enumerate([40000, 12000])]
        got = model.embed_batch(clips)
        for i, c in enumerate(clips):
            assert _cos(got[i], _oracle(mq, c)) >= COS_TOL, i
    finally:
        model.close()
