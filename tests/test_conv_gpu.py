"""GPU parity of the tcgen05 implicit-GEMM conv (vdb_conv) through the C ABI.

Oracle: the reference's blocked direct conv (src/directconv.cpp) via the C
restatement in oracle/ (pinned bit-exact to the reference's compiled kernels in
tests/test_oracle.py) on the same f16-rounded inputs/weights widened to f32.
Larger shapes use torch fp32 CPU conv2d (TF32 off) on the same values.

Tolerance (written here, per the benchmark spec): rel-L2 <= 1e-3 over valid
pixels, and every padded / masked pixel exactly 0.
"""
import numpy as np
import pytest

REL_L2_TOL = 1e-3

pytestmark = pytest.mark.gpu


def _ref_conv(x, w, bias, stride, *, x1=None, w1=None, stride1=1, residual=None, relu=False,
              clamp_hi=0.0, tvalid_out=None, use_oracle=False):
    """f32 reference on CPU: x (B,C,F,T) torch, w (OC,IC,k,k) torch."""
    import torch
    import torch.nn.functional as Fn
    import oracle
    k = w.shape[-1]
    if use_oracle:
        ys = []
        for b in range(x.shape[0]):
            ys.append(torch.from_numpy(oracle.conv2d(x[b].numpy(), w.numpy(), stride)))
        y = torch.stack(ys)
        if x1 is not None:
            y = y + torch.stack([torch.from_numpy(oracle.conv2d(x1[b].numpy(), w1.numpy(),
                                                                stride1))
                                 for b in range(x.shape[0])])
    else:
        y = Fn.conv2d(x, w, stride=stride, padding=(k - 1) // 2)
        if x1 is not None:
            y = y + Fn.conv2d(x1, w1, stride=stride1)
    y = y + bias.view(1, -1, 1, 1)
    if residual is not None:
        y = y + residual
    if relu:
        y = y.clamp_min(0)
    if clamp_hi > 0:
        y = y.clamp_max(clamp_hi)
    if tvalid_out is not None:
        for b, tv in enumerate(tvalid_out):
            y[b, :, :, int(tv):] = 0
    return y


def _h(t):
    return t.half().float()


def valid_tilings(IC, OC, k, stride, two_segments=False):
    """Every explicit (tile_m, halo, ksplit) the kernel accepts for this layer
    (tall HALO tiles may still be refused when two stages do not fit in shared
    memory; the test skips those)."""
    bn = OC if OC <= 256 else OC // ((OC + 255) // 256)
    kb = 64 if IC % 64 == 0 else (32 if IC % 32 == 0 else 16)
    ks = kb // 16
    hs_ok = k == 3 and stride == 1 and OC <= 256
    # the resident-weight halo also feeds stride-2 3x3 convs (one halo per PHASE plane)
    halo_ok = k == 3 and stride in (1, 2) and OC <= 256 and 9 * IC * bn * 2 <= 96 * 1024
    out = []
    for tile_m in (128, 256):
        nmb = tile_m // 128
        for J in (1, 2, 4, 8):
            if nmb * J * bn > 512:
                continue
            if J <= ks:
                out.append((tile_m, -1, J))
                if hs_ok:
                    out.append((tile_m, 2, J))  # streamed-weights halo (two rings)
            if halo_ok:
                out.append((tile_m, 1, J))
    if halo_ok:
        for tile_m in (384, 512, 1024):
            if tile_m // 128 * bn <= 512:
                out.append((tile_m, 1, 1))
    if bn % 32 == 0:
        out.append((256, -1, 1, 1))  # CTA pair (cta_group::2), one tap per stage
    return out


CASES = [
    # name, B, IC, OC, F, T, k, stride, fused_down, residual, tvalid_frac
    ("gemm1x1", 2, 64, 64, 8, 12, 1, 1, False, False, None),
    ("test_blocked_s1", 1, 32, 64, 11, 20, 3, 1, False, False, None),
    ("test_blocked_s2", 1, 64, 128, 11, 20, 3, 2, False, False, None),
    ("ic16_oc16", 2, 16, 16, 5, 7, 3, 1, False, False, None),
    ("s1_128_256", 2, 128, 256, 10, 38, 3, 1, False, False, None),
    ("s1_256_256", 2, 256, 256, 10, 38, 3, 1, False, True, None),
    ("s1_32_32_res", 3, 32, 32, 80, 30, 3, 1, False, True, [30, 17, 5]),
    ("s2_32_64_down", 3, 32, 64, 80, 31, 3, 2, True, False, [31, 20, 9]),
    ("oc512_split", 1, 64, 512, 6, 9, 3, 1, False, False, None),
    ("s2_1x1", 2, 64, 128, 20, 31, 1, 2, False, False, [31, 12]),
    ("s2_1x1_down", 2, 32, 64, 20, 31, 1, 2, True, False, [31, 12]),
    # large enough for the automatic choice of tall HALO tiles (8 and 3 row blocks)
    ("tall_32_32", 16, 32, 32, 80, 300, 3, 1, False, True,
     [300, 299, 251, 200, 150, 100, 64, 33, 300, 17, 9, 5, 3, 2, 1, 280]),
    ("tall_64_64", 48, 64, 64, 40, 150, 3, 1, False, False, None),
    # tall HALO tiles followed by a 1x1 segment (the identity-shortcut form)
    ("tall_32_seg1", 16, 32, 32, 80, 300, 3, 1, True, False,
     [300, 299, 251, 200, 150, 100, 64, 33, 300, 17, 9, 5, 3, 2, 1, 280]),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_conv_vs_reference(cuda_lib, case):
    import torch
    vd = cuda_lib
    name, B, IC, OC, F, T, k, stride, fused_down, use_res, tv = case
    g = torch.Generator().manual_seed(1234)
    dev = "cuda"
    x = torch.relu(torch.randn(B, IC, F, T, generator=g))
    tvalid_in = tv if tv is not None else [T] * B
    for b, t in enumerate(tvalid_in):
        x[b, :, :, t:] = 0
    w = torch.randn(OC, IC, k, k, generator=g) * (2.0 / (IC * k * k)) ** 0.5
    bias = torch.randn(OC, generator=g) * 0.1
    x, w = _h(x), _h(w)
    To, Fo = vd.out_extent(T, stride), vd.out_extent(F, stride)
    tvalid_out = [vd.out_extent(t, stride) for t in tvalid_in]
    tv_dev = torch.tensor(tvalid_out, dtype=torch.int32, device=dev)

    kw = {}
    x1 = w1 = None
    if fused_down:
        w1 = _h(torch.randn(OC, IC, 1, 1, generator=g) * (2.0 / IC) ** 0.5)
        x1 = x
        kw.update(x1=vd.to_phase(x.to(dev), tvalid_in) if stride == 2 else vd.to_grid(
            x.to(dev), tvalid_in), w1=w1.reshape(OC, IC).half().to(dev).contiguous(),
            stride1=stride)
    residual = None
    if use_res:
        residual = _h(torch.randn(B, OC, Fo, To, generator=g))
        for b, t in enumerate(tvalid_out):
            residual[b, :, :, t:] = 0
        kw["residual"] = vd.to_grid(residual.to(dev), tvalid_out)

    xin = vd.to_phase(x.to(dev), tvalid_in) if stride == 2 else vd.to_grid(x.to(dev), tvalid_in)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    small = B * OC * Fo * To * IC * k * k < 2e7
    ref = _ref_conv(x, w, bias, stride, x1=x1, w1=w1, stride1=stride, residual=residual,
                    relu=True, tvalid_out=tvalid_out, use_oracle=small)
    # every tiling the kernel offers: automatic, 128/256-row tiles, and the
    # shared-halo feed where the layer qualifies (3x3 stride 1 or 2, resident weights)
    configs = [(0, 0, 0)] + valid_tilings(IC, OC, k, stride, two_segments=fused_down)
    wp = vd.pack_conv_weight(w.to(dev))
    for cfg in configs:
        tile_m, halo, ksplit = cfg[:3]
        pair = cfg[3] if len(cfg) > 3 else 0
        try:
            y = vd.conv(xin, wp, bias.float().to(dev), tv_dev, batch=B, t_out=To, f_out=Fo,
                        oc=OC, k0=k, stride0=stride, ic0=IC, relu=True, err=err, tile_m=tile_m,
                        halo=halo, ksplit=ksplit, pair=pair, **kw)
        except RuntimeError as e:
            if tile_m > 256 and "does not fit" in str(e):
                continue
            raise
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"kernel error word {err.item():#x}"
        got = vd.from_grid(y, B, OC, Fo, To).cpu()
        rel = float((got - ref).norm() / max(ref.norm(), 1e-12))
        assert rel <= REL_L2_TOL, \
            f"{name} tile_m={tile_m} halo={halo} ksplit={ksplit} pair={pair}: rel-L2 {rel:.3e}"
        # borders and masked rows are exactly zero
        gfull = y.reshape(B, To + 2, Fo + 2, OC).float().cpu()
        assert torch.all(gfull[:, 0] == 0) and torch.all(gfull[:, :, 0] == 0)
        assert torch.all(gfull[:, :, Fo + 1] == 0)
        for b, t in enumerate(tvalid_out):
            assert torch.all(gfull[b, 1 + t:] == 0)


def test_conv_phase_output(cuda_lib):
    """y_phase=1 writes exactly the PHASE layout of the plain output."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(7)
    B, IC, OC, F, T = 2, 64, 64, 40, 21
    tv = [21, 12]
    x = torch.relu(torch.randn(B, IC, F, T, generator=g))
    for b, t in enumerate(tv):
        x[b, :, :, t:] = 0
    w = _h(torch.randn(OC, IC, 3, 3, generator=g) * 0.05)
    bias = torch.randn(OC, generator=g) * 0.1
    tvd = torch.tensor(tv, dtype=torch.int32, device="cuda")
    xin = vd.to_grid(x.cuda(), tv)
    wp = vd.pack_conv_weight(w.cuda())
    y_plain = vd.conv(xin, wp, bias.cuda(), tvd, batch=B, t_out=T, f_out=F, oc=OC, relu=True)
    y_ph = vd.conv(xin, wp, bias.cuda(), tvd, batch=B, t_out=T, f_out=F, oc=OC, relu=True,
                   y_phase=True)
    torch.cuda.synchronize()
    plain = vd.from_grid(y_plain, B, OC, F, T)
    back = vd.from_phase(y_ph, B, OC, F, T)
    assert torch.equal(plain.cpu(), back.cpu())


def _rand_act(g, B, C_, F, T, tv):
    import torch
    x = _h(torch.relu(torch.randn(B, C_, F, T, generator=g)))
    for b, t in enumerate(tv):
        x[b, :, :, t:] = 0
    return x


def _rel(got, ref):
    return float((got - ref).norm() / max(ref.norm(), 1e-12))


@pytest.mark.parametrize("k,stride", [(3, 1), (1, 1), (3, 2)])
def test_conv_channel_slices(cuda_lib, k, stride):
    """x0, residual and y as channel slices of wider GRID/PHASE tensors (the Res2Net
    width split and the channel concat, src/encoder_eres2net.cpp:108-135): results
    match the dense call, and channels outside the output slice are untouched."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(31)
    B, CW, F, T = 2, 96, 20, 23
    c0, IC, OC, o0 = 32, 32, 32, 64  # input slice [32, 64), output slice [64, 96)
    tv = [23, 14]
    To, Fo = vd.out_extent(T, stride), vd.out_extent(F, stride)
    tvo = [vd.out_extent(t, stride) for t in tv]
    xw = _rand_act(g, B, CW, F, T, tv)
    w = _h(torch.randn(OC, IC, k, k, generator=g) * (2.0 / (IC * k * k)) ** 0.5)
    bias = torch.randn(OC, generator=g) * 0.1
    res_w = _rand_act(g, B, CW, Fo, To, tvo)
    tvd = torch.tensor(tvo, dtype=torch.int32, device="cuda")
    to_l = vd.to_phase if stride == 2 else vd.to_grid
    xin = to_l(xw.cuda(), tv)
    rin = vd.to_grid(res_w.cuda(), tvo)
    wp = vd.pack_conv_weight(w.cuda())
    sentinel = 3.0
    yw = torch.full((vd.lib().vdb_grid_rows(B, To, Fo), CW), sentinel, dtype=torch.float16,
                    device="cuda")
    vd.conv(xin[:, c0:c0 + IC], wp, bias.cuda(), tvd, batch=B, t_out=To, f_out=Fo, oc=OC, k0=k,
            stride0=stride, ic0=IC, residual=rin[:, o0:o0 + OC], relu=True,
            y=yw[:, o0:o0 + OC])
    torch.cuda.synchronize()
    ref = _ref_conv(xw[:, c0:c0 + IC], w, bias, stride, residual=res_w[:, o0:o0 + OC],
                    relu=True, tvalid_out=tvo)
    got = vd.from_grid(yw[:, o0:o0 + OC].contiguous(), B, OC, Fo, To).cpu()
    assert _rel(got, ref) <= REL_L2_TOL
    assert torch.all(yw[:, :o0].float() == sentinel)


def test_conv_dual_output(cuda_lib):
    """y2 receives the PHASE layout of the same values y gets in GRID layout."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(32)
    B, IC, OC, F, T = 2, 64, 128, 40, 33
    tv = [33, 18]
    x = _rand_act(g, B, IC, F, T, tv)
    w = _h(torch.randn(OC, IC, 3, 3, generator=g) * 0.05)
    bias = torch.randn(OC, generator=g) * 0.1
    tvd = torch.tensor(tv, dtype=torch.int32, device="cuda")
    xin = vd.to_grid(x.cuda(), tv)
    wp = vd.pack_conv_weight(w.cuda())
    y2 = torch.zeros(vd.lib().vdb_phase_rows(B, T, F), OC, dtype=torch.float16, device="cuda")
    y = vd.conv(xin, wp, bias.cuda(), tvd, batch=B, t_out=T, f_out=F, oc=OC, relu=True, y2=y2)
    torch.cuda.synchronize()
    plain = vd.from_grid(y, B, OC, F, T).cpu()
    assert torch.equal(plain, vd.from_phase(y2, B, OC, F, T).cpu())
    ref = _ref_conv(x, w, bias, 1, relu=True, tvalid_out=tv)
    assert _rel(plain, ref) <= REL_L2_TOL


def test_conv_silu_no_bias(cuda_lib):
    """act=1: SiLU(conv) with no bias (the AFF local_att first conv + SiLU,
    src/encoder_eres2net.cpp:64-67, with bias=NULL accepted)."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(33)
    B, IC, OC, F, T = 2, 128, 32, 10, 19
    tv = [19, 7]
    x = _h(torch.randn(B, IC, F, T, generator=g))
    for b, t in enumerate(tv):
        x[b, :, :, t:] = 0
    w = _h(torch.randn(OC, IC, 1, 1, generator=g) * (1.0 / IC) ** 0.5)
    tvd = torch.tensor(tv, dtype=torch.int32, device="cuda")
    y = vd.conv(vd.to_grid(x.cuda(), tv), vd.pack_conv_weight(w.cuda()), None, tvd, batch=B,
                t_out=T, f_out=F, oc=OC, k0=1, act=1)
    torch.cuda.synchronize()
    lin = _ref_conv(x, w, torch.zeros(OC), 1)
    ref = lin * torch.sigmoid(lin)
    for b, t in enumerate(tv):
        ref[b, :, :, t:] = 0
    assert _rel(vd.from_grid(y, B, OC, F, T).cpu(), ref) <= REL_L2_TOL


def test_conv_attentional_fusion(cuda_lib):
    """act=2: (x + ds) + tanh(conv(z) + b) * (x - ds), the AFF output
    (src/encoder_eres2net.cpp:69-75), with x / ds / y as channel slices."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(34)
    B, IC, OC, F, T = 2, 32, 128, 10, 17
    tv = [17, 9]
    z = _h(torch.randn(B, IC, F, T, generator=g))
    for b, t in enumerate(tv):
        z[b, :, :, t:] = 0
    xw = _rand_act(g, B, 2 * OC, F, T, tv)   # x in channels [0, OC), ds in [OC, 2 OC)
    w = _h(torch.randn(OC, IC, 1, 1, generator=g) * (1.0 / IC) ** 0.5)
    bias = torch.randn(OC, generator=g) * 0.1
    tvd = torch.tensor(tv, dtype=torch.int32, device="cuda")
    xg = vd.to_grid(xw.cuda(), tv)
    y = vd.conv(vd.to_grid(z.cuda(), tv), vd.pack_conv_weight(w.cuda()), bias.cuda(), tvd,
                batch=B, t_out=T, f_out=F, oc=OC, k0=1, residual=xg[:, :OC],
                residual2=xg[:, OC:], act=2)
    torch.cuda.synchronize()
    att = torch.tanh(_ref_conv(z, w, bias, 1))
    xa, ds = xw[:, :OC], xw[:, OC:]
    ref = (xa + ds) + att * (xa - ds)
    for b, t in enumerate(tv):
        ref[b, :, :, t:] = 0
    assert _rel(vd.from_grid(y, B, OC, F, T).cpu(), ref) <= REL_L2_TOL


def test_add_slices(cuda_lib):
    """vdb_add on channel slices is exact f16(a + b) and leaves other channels alone."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(35)
    rows = 1000
    a = torch.randn(rows, 64, generator=g).half().cuda()
    b = torch.randn(rows, 48, generator=g).half().cuda()
    y = torch.full((rows, 80), 7.0, dtype=torch.float16, device="cuda")
    vd.add(a[:, 16:48], b[:, 8:40], y[:, 40:72])
    torch.cuda.synchronize()
    ref = (a[:, 16:48].float() + b[:, 8:40].float()).half()
    assert torch.equal(y[:, 40:72], ref)
    assert torch.all(y[:, :40] == 7.0) and torch.all(y[:, 72:] == 7.0)


def test_conv_sum_output(cuda_lib):
    """ysum = f16(y + addend) from the epilogue, on channel slices, equal bit for bit to
    a separate vdb_add of the stored y (the fused Res2Net `sp + chunk`)."""
    import torch
    vd = cuda_lib
    g = torch.Generator().manual_seed(36)
    B, IC, OC, F, T = 2, 32, 32, 40, 27
    tv = [27, 11]
    x = _rand_act(g, B, IC, F, T, tv)
    w = _h(torch.randn(OC, IC, 3, 3, generator=g) * 0.1)
    bias = torch.randn(OC, generator=g) * 0.1
    tvd = torch.tensor(tv, dtype=torch.int32, device="cuda")
    xin = vd.to_grid(x.cuda(), tv)
    wide = vd.to_grid(_rand_act(g, B, 3 * OC, F, T, tv).cuda(), tv)  # addend = channels [OC, 2 OC)
    rows = vd.lib().vdb_grid_rows(B, T, F)
    ys = torch.full((rows, 2 * OC), 5.0, dtype=torch.float16, device="cuda")
    y = vd.conv(xin, vd.pack_conv_weight(w.cuda()), bias.cuda(), tvd, batch=B, t_out=T, f_out=F,
                oc=OC, relu=True, clamp_hi=20.0, ysum=ys[:, OC:], addend=wide[:, OC:2 * OC])
    ref = vd.add(y, wide[:, OC:2 * OC])
    torch.cuda.synchronize()
    assert torch.equal(ys[:, OC:], ref)
    assert torch.all(ys[:, :OC] == 5.0)
    g4 = ys[:, OC:].reshape(B, T + 2, F + 2, OC).float()
    assert torch.all(g4[:, 0] == 0) and torch.all(g4[:, :, 0] == 0)
    for b, t in enumerate(tv):
        assert torch.all(g4[b, 1 + t:] == 0)


QPACK_CASES = [
    # name, B, F, T, tvalid, residual, y_phase, tile_m
    ("qp_ragged", 3, 80, 37, [37, 20, 5], False, 0, 0),
    ("qp_res", 3, 80, 37, [37, 21, 1], True, 0, 0),
    ("qp_phase", 2, 80, 31, [31, 12], True, 1, 0),
    ("qp_tile128", 3, 80, 37, [37, 20, 5], True, 0, 128),
    ("qp_tall", 16, 80, 300, [300, 299, 251, 200, 150, 100, 64, 33, 300, 17, 9, 5, 3, 2, 1, 280],
     True, 0, 0),
    ("qp_f16", 4, 16, 23, [23, 9, 1, 14], True, 0, 0),
    ("qp_f18_phase", 2, 18, 9, [9, 4], False, 1, 128),
]


@pytest.mark.parametrize("case", QPACK_CASES, ids=[c[0] for c in QPACK_CASES])
def test_conv_qpack_vs_reference(cuda_lib, case):
    """Stage-1 conv over the QPACK layout (four frequency pixels per row, the
    (time tap, pixel shift) MMA schedule) against the f32 conv of the same f16 values:
    rel-L2 <= 1e-3 over valid pixels, exact zeros at borders, past each clip's length
    and past the padded grid; optional QPACK residual (the BasicBlock identity) and the
    PHASE output of the last stage-1 conv."""
    import torch
    vd = cuda_lib
    name, B, F, T, tv, use_res, y_phase, tile_m = case
    g = torch.Generator().manual_seed(99)
    x = _h(torch.relu(torch.randn(B, 32, F, T, generator=g)))
    for b, t in enumerate(tv):
        x[b, :, :, t:] = 0
    w = _h(torch.randn(32, 32, 3, 3, generator=g) * (2.0 / (32 * 9)) ** 0.5)
    bias = torch.randn(32, generator=g) * 0.1
    res = None
    if use_res:
        res = _h(torch.relu(torch.randn(B, 32, F, T, generator=g)))
        for b, t in enumerate(tv):
            res[b, :, :, t:] = 0
    ref = _ref_conv(x, w, bias, 1, residual=res, relu=True, tvalid_out=tv,
                    use_oracle=B * 32 * F * T * 288 < 2e7)
    dev = "cuda"
    tv_dev = torch.tensor(tv, dtype=torch.int32, device=dev)
    wq = vd.qpack_weights(vd.pack_conv_weight(w.to(dev)))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    y = vd.conv(vd.to_qpack(x.to(dev), tv), wq, bias.float().to(dev), tv_dev, batch=B, t_out=T,
                f_out=F, oc=32, k0=3, ic0=32, relu=True, err=err, tile_m=tile_m, qpack=True,
                residual=vd.to_qpack(res.to(dev), tv) if use_res else None, y_phase=y_phase)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    if y_phase:
        got = vd.from_phase(y, B, 32, F, T).cpu()
    else:
        got = vd.from_qpack(y, B, F, T).cpu()
        full = vd.from_qpack(y, B, F, T, interior=False).cpu()  # (B, 32, 4Wq, T+2)
        assert torch.all(full[:, :, :, 0] == 0) and torch.all(full[:, :, 0] == 0)
        assert torch.all(full[:, :, F + 1:] == 0)  # right border and past the grid
        for b, t in enumerate(tv):
            assert torch.all(full[b, :, :, 1 + t:] == 0)
    rel = float((got - ref).norm() / max(ref.norm(), 1e-12))
    assert rel <= REL_L2_TOL, f"{name}: rel-L2 {rel:.3e}"


Q8_CASES = [
    # name, B, IC, OC, F, T, stride, second segment ("down" 1x1 s2 / "id" / None), kwargs
    ("halo_resident_64", 3, 64, 64, 20, 24, 1, None, {}),
    ("halo_streamed_128", 3, 128, 128, 10, 20, 1, None, {}),
    ("pair_256", 3, 256, 256, 10, 12, 1, None, {}),
    ("tap_s2_32_64", 3, 32, 64, 40, 30, 2, None, {}),
    ("tap_forced_64", 3, 64, 64, 20, 24, 1, None, {"halo": -1}),
    ("down_64", 3, 64, 64, 20, 24, 1, "down", {}),
    ("id_128_mixed", 3, 128, 128, 10, 20, 1, "id", {}),
    ("halo_s2_32_64", 3, 32, 64, 40, 30, 2, None, {"halo": 1}),
    # several tiles per CTA: stages reused across tiles by q8_0 and f16 segments
    ("id_128_multi", 64, 128, 128, 20, 75, 1, "id", {}),
    ("pair_id_256_multi", 256, 256, 256, 10, 38, 1, "id", {}),
    ("down_64_multi", 64, 64, 64, 40, 150, 1, "down", {}),
    ("tap_s2_64_128_multi", 64, 64, 128, 40, 150, 2, None, {}),
    ("down_256_pair_multi", 256, 256, 256, 10, 38, 1, "down", {}),
]


@pytest.mark.parametrize("case", Q8_CASES, ids=[c[0] for c in Q8_CASES])
def test_conv_q8_weights_equal_their_f16_expansion(cuda_lib, case):
    """q8_0 weights (int8 values + an f16 scale per 32 input channels) expanded in
    shared memory give bit-identical outputs to the same conv fed the f16 weights
    f16(q * d): every weight feed (resident halo, streamed halo, CTA pairs, one tap per
    stage, the 1x1 downsample segment; an f16 identity segment beside a q8_0 one)."""
    import torch
    vd = cuda_lib
    name, B, IC, OC, F, T, stride, seg1, kw = case
    g = torch.Generator().manual_seed(7)
    dev = "cuda"
    To, Fo = vd.out_extent(T, stride), vd.out_extent(F, stride)
    tv = ([To, max(1, To // 2), 1] * B)[:B]
    x = _h(torch.relu(torch.randn(B, IC, F, T, generator=g)))
    xg = (vd.to_phase if stride == 2 else vd.to_grid)(x.to(dev))
    w = torch.randn(OC, 9, IC, generator=g) * (2.0 / (9 * IC)) ** 0.5
    q, d, w16 = vd.q8_planes(w.to(dev))
    bias = (torch.randn(OC, generator=g) * 0.1).to(dev)
    tvd = torch.tensor(tv, dtype=torch.int32, device=dev)
    extra_f16, extra_q8 = {}, {}
    if seg1 == "down":
        x1 = vd.to_phase(_h(torch.relu(torch.randn(B, IC // 2, 2 * Fo, 2 * To, generator=g))).to(dev))
        w1 = torch.randn(OC, IC // 2, generator=g) * 0.1
        q1, d1, w1_16 = vd.q8_planes(w1.to(dev))
        extra_f16 = dict(x1=x1, w1=w1_16, stride1=2)
        extra_q8 = dict(x1=x1, w1=q1, w1_scale=d1, stride1=2)
    elif seg1 == "id":
        x1 = vd.to_grid(_h(torch.relu(torch.randn(B, OC, Fo, To, generator=g))).to(dev))
        eye = torch.eye(OC, device=dev).half()
        extra_f16 = dict(x1=x1, w1=eye, stride1=1)
        extra_q8 = dict(x1=x1, w1=eye, stride1=1)
    args = dict(batch=B, t_out=To, f_out=Fo, oc=OC, k0=3, stride0=stride, ic0=IC, relu=True, **kw)
    y16 = vd.conv(xg, w16, bias, tvd, **args, **extra_f16)
    y8 = vd.conv(xg, q, bias, tvd, w0_scale=d, **args, **extra_q8)
    torch.cuda.synchronize()
    assert torch.equal(y8, y16), (name, (y8.float() - y16.float()).abs().max().item())
    assert y16.float().abs().sum().item() > 0


def test_conv_qpack_q8_weights_equal_their_f16_expansion(cuda_lib):
    """The QPACK stage-1 conv with q8_0 packed weights (expanded once per CTA) equals
    the same conv on the f16 packed weights, with the residual and both outputs."""
    import torch
    vd = cuda_lib
    B, F, T, dev = 4, 80, 41, "cuda"
    g = torch.Generator().manual_seed(11)
    tv = torch.tensor([41, 30, 7, 1], dtype=torch.int32, device=dev)
    x = vd.to_qpack(_h(torch.relu(torch.randn(B, 32, F, T, generator=g))).to(dev))
    r = vd.to_qpack(_h(torch.relu(torch.randn(B, 32, F, T, generator=g))).to(dev))
    w = torch.randn(32, 9, 32, generator=g) * (2.0 / 288) ** 0.5
    q, d, w16 = vd.q8_planes(w.to(dev))
    wq16 = vd.qpack_weights(w16)
    qq, dq = vd.qpack_q8(q, d)
    bias = (torch.randn(32, generator=g) * 0.1).to(dev)
    L = vd.lib()
    for y_phase in (0, 1):
        kw = dict(batch=B, t_out=T, f_out=F, oc=32, k0=3, ic0=32, relu=True, qpack=True,
                  residual=r, y_phase=y_phase)
        # the PHASE output has slots the conv never writes: start both from zeros
        shape = (L.vdb_phase_rows(B, T, F), 32) if y_phase else tuple(x.shape)
        y16 = vd.conv(x, wq16, bias, tv, y=torch.zeros(shape, dtype=torch.float16, device=dev), **kw)
        y8 = vd.conv(x, qq, bias, tv, w0_scale=dq,
                     y=torch.zeros(shape, dtype=torch.float16, device=dev), **kw)
        torch.cuda.synchronize()
        assert torch.equal(y8, y16), y_phase


def test_conv_q8_rejects_bad_channel_counts(cuda_lib):
    import torch
    vd = cuda_lib
    dev = "cuda"
    x = torch.zeros(vd.lib().vdb_grid_rows(1, 8, 8), 16, dtype=torch.float16, device=dev)
    q = torch.zeros(16, 9, 16, dtype=torch.int8, device=dev)
    d = torch.ones(16, 9, 1, dtype=torch.float16, device=dev)
    tv = torch.tensor([8], dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        vd.conv(x, q, None, tv, batch=1, t_out=8, f_out=8, oc=16, k0=3, ic0=16, w0_scale=d)
