"""vdb_cmn_stem_noalloc: the CMN + stem entry point for callers that cannot
allocate device memory (a streaming audio callback that must not stall on
cudaMalloc, or a host that owns every device allocation through its own pool).

It keeps the per-clip CMN means in a fixed array inside the library instead of
caller-provided working memory. Checked through the C ABI against the existing
entry point, vdb_cmn_stem, on two calls in a row with different inputs (so a
stale array would show), directly against the CPU oracle's CMN + stem conv at
rel-L2 <= 1e-3 (with and without CMN, 16 / 32 / 64 stem channels), and for its
size limit. The file name sorts last so that a run stopping at the first failure
has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(seed, B, t_max, frames, M=80, OC=32):
    import torch
    rng = np.random.default_rng(seed)
    feats = torch.from_numpy(rng.standard_normal((B, t_max, M)).astype(np.float32) * 3 + 1).cuda()
    fr = torch.tensor(frames, dtype=torch.int32, device="cuda")
    w = torch.from_numpy((rng.standard_normal((OC, 9)) * 0.4).astype(np.float32)).cuda()
    b = torch.from_numpy((rng.standard_normal(OC) * 0.1).astype(np.float32)).cuda()
    return feats, fr, w, b


def _run_both(vd, feats, fr, w, b, B, t_max, M=80, OC=32, cmn=1):
    import torch
    L = vd.lib()
    rows = L.vdb_grid_rows(B, t_max, M)
    y_ref = torch.full((rows, OC), 7.0, dtype=torch.float16, device="cuda")
    y_new = torch.full((rows, OC), -7.0, dtype=torch.float16, device="cuda")
    scratch = torch.empty(B, M, device="cuda")
    rc = L.vdb_cmn_stem(feats.data_ptr(), fr.data_ptr(), B, t_max, M, cmn, w.data_ptr(),
                        b.data_ptr(), OC, scratch.data_ptr(), y_ref.data_ptr(), None)
    assert rc == 0, vd.last_error()
    rc = L.vdb_cmn_stem_noalloc(feats.data_ptr(), fr.data_ptr(), B, t_max, M, cmn, w.data_ptr(),
                                b.data_ptr(), OC, y_new.data_ptr(), None)
    assert rc == 0, vd.last_error()
    torch.cuda.synchronize()
    return y_ref, y_new


def test_noalloc_matches_allocating_entry_point_twice(cuda_lib):
    import torch
    # first call: 3 ragged clips
    feats, fr, w, b = _inputs(1, 3, 41, [41, 17, 2])
    y_ref, y_new = _run_both(cuda_lib, feats, fr, w, b, 3, 41)
    rel = float((y_new.float() - y_ref.float()).norm() / y_ref.float().norm())
    assert rel <= 1e-3 and torch.equal(y_new, y_ref)
    # second call in a row: different batch, lengths and values
    feats, fr, w, b = _inputs(2, 5, 23, [23, 23, 9, 1, 14])
    y_ref, y_new = _run_both(cuda_lib, feats, fr, w, b, 5, 23)
    rel = float((y_new.float() - y_ref.float()).norm() / y_ref.float().norm())
    assert rel <= 1e-3 and torch.equal(y_new, y_ref)


@pytest.mark.parametrize("oc,cmn", [(16, 1), (32, 0), (64, 1)])
def test_noalloc_matches_oracle(cuda_lib, oc, cmn):
    """Against the CPU oracle directly: per-clip CMN over each clip's valid frames
    (src/fbank.cpp:194-201, skipped when cmn = 0), then the 3x3 stem conv + bias +
    ReLU (src/encoder_resnet.cpp:116-117), rel-L2 <= 1e-3 per clip, zeros past each
    clip's valid length."""
    import oracle
    B, t_max, M = 4, 29, 80
    frames = [29, 11, 1, 20]
    feats, fr, w, b = _inputs(10 + oc + cmn, B, t_max, frames, M, oc)
    _, y_new = _run_both(cuda_lib, feats, fr, w, b, B, t_max, M, oc, cmn)
    got = cuda_lib.from_grid(y_new, B, oc, M, t_max).cpu().numpy()
    x_all = feats.cpu().numpy()
    # [oc][9] taps kt*3 + kf (kt = time, kf = freq) -> torch layout (oc, 1, freq, time)
    w4 = w.cpu().numpy().reshape(oc, 3, 3).transpose(0, 2, 1)[:, None].copy()
    bias = b.cpu().numpy()
    for i, T in enumerate(frames):
        x = x_all[i, :T, :].T.copy()  # [80, T] feat-major
        if cmn:
            x -= (x.astype(np.float64).sum(1, keepdims=True) / T).astype(np.float32)
        want = oracle.conv2d(x[None], w4, 1, bias, True)
        have = got[i, :, :, :T]
        rel = np.linalg.norm(have - want) / max(np.linalg.norm(want), 1e-12)
        assert rel <= 1e-3, (i, rel)
        assert np.all(got[i, :, :, T:] == 0)


def test_noalloc_rejects_oversized_batch(cuda_lib):
    L = cuda_lib.lib()
    # 820 clips x 80 mels = 65600 means > 65536: rejected before any work
    rc = L.vdb_cmn_stem_noalloc(1, 1, 820, 10, 80, 1, 1, 1, 32, 1, None)
    assert rc != 0
    assert "65536" in cuda_lib.last_error()
