"""BASELINE config 1, per layer: every distinct ResNet34 conv shape at its configured
extent (T = 300 frames, 80 mel bins in; batch 4), checked against the reference's
own kernels compiled unmodified in oracle/_ref:

* the blocked direct conv (src/directconv.cpp:1496-1522, blocked_conv3x3 /
  blocked_conv1x1) for every shape, and
* the Winograd conv (src/winograd.cpp:638-648, winograd_conv3x3, stride 1 only)
  for every stride-1 3x3 shape, and the NCHW direct conv (directconv_conv3x3,
  src/directconv.cpp:1449-1458) for the 1-channel stem.

Activations ReLU(N(0, 1)) in f16, weights f16 Kaiming-normal, both widened to f32
for the reference; the GPU accumulates in f32. Gate: rel-L2 <=
1e-3 over the valid output, per layer and per reference kernel.
"""
import zlib

import numpy as np
import pytest

import oracle

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ref_available(),
                                 reason="oracle/_ref (the reference compiled) not built")]

REL_L2_TOL = 1e-3
B = 4

# (name, IC, OC, F_in, T_in, k, stride) -- the 11 distinct shapes of the net
SHAPES = [
    ("stem_1_32", 1, 32, 80, 300, 3, 1),
    ("s1_32_32", 32, 32, 80, 300, 3, 1),
    ("s2_32_64", 32, 64, 80, 300, 3, 2),
    ("down_32_64", 32, 64, 80, 300, 1, 2),
    ("s1_64_64", 64, 64, 40, 150, 3, 1),
    ("s2_64_128", 64, 128, 40, 150, 3, 2),
    ("down_64_128", 64, 128, 40, 150, 1, 2),
    ("s1_128_128", 128, 128, 20, 75, 3, 1),
    ("s2_128_256", 128, 256, 20, 75, 3, 2),
    ("down_128_256", 128, 256, 20, 75, 1, 2),
    ("s1_256_256", 256, 256, 10, 38, 3, 1),
]


def _rel(got, want):
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-12))


@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
def test_config1_layer_vs_reference_kernels(cuda_lib, shape):
    import torch
    vd = cuda_lib
    name, IC, OC, F, T, k, stride = shape
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    x = torch.relu(torch.randn(B, IC, F, T, generator=g)).half().float()
    w = (torch.randn(OC, IC, k, k, generator=g) * (2.0 / (IC * k * k)) ** 0.5).half().float()
    To, Fo = vd.out_extent(T, stride), vd.out_extent(F, stride)
    tv = torch.tensor([To] * B, dtype=torch.int32, device="cuda")
    if IC == 1:
        # the stem: f32 features through the CMN + stem kernel with CMN off and a zero
        # bias (features [B, T, 80] frame-major, weights [OC][9] with tap kt*3 + kf)
        L = vd.lib()
        feats = x[:, 0].permute(0, 2, 1).contiguous().cuda()
        frames = torch.tensor([T] * B, dtype=torch.int32, device="cuda")
        w9 = w[:, 0].permute(0, 2, 1).reshape(OC, 9).contiguous().cuda()
        zero = torch.zeros(OC, device="cuda")
        means = torch.empty(B, F, device="cuda")
        y = torch.empty(L.vdb_grid_rows(B, T, F), OC, dtype=torch.float16, device="cuda")
        rc = L.vdb_cmn_stem(feats.data_ptr(), frames.data_ptr(), B, T, F, 0, w9.data_ptr(),
                            zero.data_ptr(), OC, means.data_ptr(), y.data_ptr(), None)
        assert rc == 0, vd.last_error()
        torch.cuda.synchronize()
        got = vd.from_grid(y, B, OC, F, T).cpu().numpy()
        # the stem applies ReLU: compare against ReLU of the references
        refs = {"directconv": lambda xb: np.maximum(oracle.ref_directconv3x3(xb, w.numpy()), 0),
                "winograd": lambda xb: np.maximum(oracle.ref_winograd3x3(xb, w.numpy()), 0)}
    else:
        xin = (vd.to_phase(x.cuda(), [T] * B) if stride == 2 else vd.to_grid(x.cuda(), [T] * B))
        if k == 3:
            wp = vd.pack_conv_weight(w.cuda())
        else:
            wp = w.reshape(OC, IC).half().cuda().contiguous()
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        y = vd.conv(xin, wp, None, tv, batch=B, t_out=To, f_out=Fo, oc=OC, k0=k,
                    stride0=stride, ic0=IC, relu=False, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = vd.from_grid(y, B, OC, Fo, To).cpu().numpy()
        wn = w.numpy()
        if k == 1:
            refs = {"directconv": lambda xb: oracle.ref_conv1x1(xb, wn, stride)}
        else:
            refs = {"directconv": lambda xb: oracle.ref_conv3x3(xb, wn, stride)}
            if stride == 1:
                refs["winograd"] = lambda xb: oracle.ref_winograd3x3(xb, wn)
    xs = x.numpy()
    for kind, fn in refs.items():
        for b in range(B):
            want = fn(xs[b])
            assert want.shape == got[b].shape, (kind, want.shape, got[b].shape)
            rel = _rel(got[b], want)
            assert rel <= REL_L2_TOL, f"{name} vs {kind}, clip {b}: rel-L2 {rel:.3e}"
