"""GPU parity of the FBank, CMN+stem and pooling kernels through the op-level C
ABI (include/vdb_ops.h), against the CPU oracle.

Tolerances: FBank max|d| <= 1e-3 (the reference's tests/test_fbank.cpp gate);
stem output within f16 rounding (rel-L2 <= 1e-3); pooled embedding cosine >=
0.9999 and pre-norm rel-L2 <= 1e-4 on the same f16 activation.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
import vd_synth

pytestmark = pytest.mark.gpu


def _fbank_plan(L):
    p = L.vdb_fbank_plan_create(16000, 80, 512, 400, 160, 0.97, 20.0, 0.0)
    assert p
    return p


def test_fbank_kernel_matches_oracle(cuda_lib):
    import torch
    L = cuda_lib.lib()
    plan = _fbank_plan(L)
    lens = [48000, 16037, 400, 399, 160000]
    clips = [vd_synth.clip_f32(vd_synth.make_clip(20 + i, n)) for i, n in enumerate(lens)]
    flat = torch.from_numpy(np.concatenate(clips)).cuda()
    offs = torch.tensor(np.cumsum([0] + lens[:-1]), dtype=torch.int64, device="cuda")
    ns = torch.tensor(lens, dtype=torch.int32, device="cuda")
    t_max = max(oracle.n_frames(n) for n in lens)
    feats = torch.full((len(lens), t_max, 80), 123.0, device="cuda")
    rc = L.vdb_fbank(plan, flat.data_ptr(), offs.data_ptr(), ns.data_ptr(), len(lens), t_max,
                     feats.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == 0, cuda_lib.last_error()
    got = feats.cpu().numpy()
    for i, c in enumerate(clips):
        T = oracle.n_frames(len(c))
        want = oracle.fbank(c, cmn=False)  # [80, T]
        assert want.shape[1] == T
        if T:
            assert np.abs(got[i, :T, :].T - want).max() <= 1e-3
        assert np.all(got[i, T:, :] == 123.0)  # frames past T_b untouched
    L.vdb_fbank_plan_destroy(plan)


def test_cmn_stem_matches_oracle(cuda_lib):
    import torch
    L = cuda_lib.lib()
    rng = np.random.default_rng(5)
    B, t_max, M, OC = 3, 37, 80, 32
    frames = [37, 20, 1]
    feats = rng.standard_normal((B, t_max, M)).astype(np.float32) * 3 + 1
    w = (rng.standard_normal((OC, 1, 3, 3)) * 0.4).astype(np.float32)
    b = (rng.standard_normal(OC) * 0.1).astype(np.float32)
    # stem weight [OC][9] with tap kt*3 + kf (kt = kw = time, kf = kh = freq)
    w_taps = np.ascontiguousarray(w[:, 0].transpose(0, 2, 1).reshape(OC, 9))
    d_feats = torch.from_numpy(feats).cuda()
    d_fr = torch.tensor(frames, dtype=torch.int32, device="cuda")
    d_w = torch.from_numpy(w_taps).cuda()
    d_b = torch.from_numpy(b).cuda()
    d_mean = torch.empty(B, M, device="cuda")
    y = torch.empty(cuda_lib.lib().vdb_grid_rows(B, t_max, M), OC, dtype=torch.float16,
                    device="cuda")
    rc = L.vdb_cmn_stem(d_feats.data_ptr(), d_fr.data_ptr(), B, t_max, M, 1, d_w.data_ptr(),
                        d_b.data_ptr(), OC, d_mean.data_ptr(), y.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == 0, cuda_lib.last_error()
    got = cuda_lib.from_grid(y, B, OC, M, t_max).cpu().numpy()
    g = y.reshape(B, t_max + 2, M + 2, OC).float().cpu().numpy()
    assert np.all(g[:, 0] == 0) and np.all(g[:, :, 0] == 0) and np.all(g[:, :, M + 1] == 0)
    for i in range(B):
        T = frames[i]
        x = feats[i, :T, :].T.copy()  # [80, T] feat-major
        x -= (x.astype(np.float64).sum(1, keepdims=True) / T).astype(np.float32)
        want = oracle.conv2d(x[None], w, 1, b, True)  # (OC, 80, T)
        have = got[i, :, :, :T]
        rel = np.linalg.norm(have - want) / max(np.linalg.norm(want), 1e-12)
        assert rel <= 1e-3
        assert np.all(got[i, :, :, T:] == 0)


@pytest.mark.parametrize("B,T,F,Cc,D", [(4, 38, 10, 256, 256), (70, 13, 10, 512, 512),
                                         (37, 9, 5, 32, 192)])
def test_pool_embed_matches_oracle(cuda_lib, B, T, F, Cc, D):
    """TSTP + split-K FC + finish/L2 vs f64 numpy; the larger cases span several
    32-clip FC tiles, several K splits and output widths that are not multiples of 64."""
    import torch
    L = cuda_lib.lib()
    rng = np.random.default_rng(8 + B)
    tv = [T, T // 2 + 1, 2, 1] + [int(v) for v in rng.integers(1, T + 1, B - 4)]
    # values exactly representable in f16, so the kernel and the f64 check see the same input
    x = (np.abs(rng.standard_normal((B, Cc, F, T))) * 5).astype(np.float16).astype(np.float32)
    for i, t in enumerate(tv):
        x[i, :, :, t:] = 0
    W = (rng.standard_normal((D, 2 * Cc * F)) / np.sqrt(2 * Cc * F)).astype(np.float32)
    bb = (rng.standard_normal(D) * 0.01).astype(np.float32)
    mv = (rng.standard_normal(D) * 0.05).astype(np.float32)
    g = cuda_lib.to_grid(torch.from_numpy(x).cuda(), tv)
    d_tv = torch.tensor(tv, dtype=torch.int32, device="cuda")
    dW, db, dmv = (torch.from_numpy(a).cuda() for a in (W, bb, mv))
    emb = torch.empty(B, D, device="cuda")
    pre = torch.empty(B, D, device="cuda")
    rc = L.vdb_pool_embed(g.data_ptr(), d_tv.data_ptr(), B, T, F, Cc, dW.data_ptr(),
                          db.data_ptr(), dmv.data_ptr(), D, 1e-8, 1, emb.data_ptr(),
                          pre.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == 0, cuda_lib.last_error()
    for i, t in enumerate(tv):
        a = x[i, :, :, :t].astype(np.float64)  # (C, F, t)
        mean = a.mean(-1)
        var = ((a - mean[..., None]) ** 2).mean(-1) * (t / (t - 1) if t > 1 else 1.0)
        pooled = np.concatenate([mean.ravel(), np.sqrt(var + 1e-8).ravel()])  # C-outer, F-inner
        e = W.astype(np.float64) @ pooled + bb - mv
        p = pre[i].cpu().numpy()
        assert np.linalg.norm(p - e) / np.linalg.norm(e) <= 1e-4
        en = e / np.linalg.norm(e)
        assert float(np.dot(emb[i].cpu().numpy(), en)) >= 0.9999


def test_cmn_stem_qpack_equals_grid(cuda_lib):
    """vdb_cmn_stem_qpack (the QPACK input of the stage-1 convs) holds exactly the
    values vdb_cmn_stem writes in the GRID layout, and zeros in every other slot
    (borders, frames past each clip, the pixels past the padded grid)."""
    import torch
    L = cuda_lib.lib()
    rng = np.random.default_rng(17)
    B, t_max, M, OC = 4, 29, 80, 32
    frames = [29, 11, 1, 20]
    feats = torch.from_numpy(rng.standard_normal((B, t_max, M)).astype(np.float32) * 3 + 1).cuda()
    fr = torch.tensor(frames, dtype=torch.int32, device="cuda")
    w = torch.from_numpy((rng.standard_normal((OC, 9)) * 0.4).astype(np.float32)).cuda()
    b = torch.from_numpy((rng.standard_normal(OC) * 0.1).astype(np.float32)).cuda()
    mean = torch.empty(B, M, device="cuda")
    yg = torch.full((L.vdb_grid_rows(B, t_max, M), OC), 3.0, dtype=torch.float16, device="cuda")
    yq = torch.full((L.vdb_qpack_rows(B, t_max, M), 128), 3.0, dtype=torch.float16, device="cuda")
    assert L.vdb_cmn_stem(feats.data_ptr(), fr.data_ptr(), B, t_max, M, 1, w.data_ptr(),
                          b.data_ptr(), OC, mean.data_ptr(), yg.data_ptr(), None) == 0
    assert L.vdb_cmn_stem_qpack(feats.data_ptr(), fr.data_ptr(), B, t_max, M, 1, w.data_ptr(),
                                b.data_ptr(), mean.data_ptr(), yq.data_ptr(), None) == 0
    torch.cuda.synchronize()
    g = yg.reshape(B, t_max + 2, M + 2, OC).permute(0, 3, 2, 1).cpu()  # (B, C, F+2, T+2)
    q = cuda_lib.from_qpack(yq, B, M, t_max, interior=False).cpu()     # (B, C, 4Wq, T+2)
    assert torch.equal(q[:, :, :M + 2], g)
    assert torch.all(q[:, :, M + 2:] == 0)
