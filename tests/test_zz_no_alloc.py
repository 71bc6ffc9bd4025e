"""vdb_cmn_stem_noalloc: the CMN + stem entry point for callers that cannot
allocate device memory (a streaming audio callback that must not stall on
cudaMalloc, or a host that owns every device allocation through its own pool).

It keeps the per-clip CMN means in a fixed array inside the library instead of
caller-provided working memory. Checked through the C ABI against the existing
entry point, vdb_cmn_stem, on two calls in a row with different inputs (so a
stale array would show), and for its size limit. The file name sorts last so
that a run stopping at the first failure has already run every other test.
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


def _run_both(vd, feats, fr, w, b, B, t_max, M=80, OC=32):
    import torch
    L = vd.lib()
    rows = L.vdb_grid_rows(B, t_max, M)
    y_ref = torch.full((rows, OC), 7.0, dtype=torch.float16, device="cuda")
    y_new = torch.full((rows, OC), -7.0, dtype=torch.float16, device="cuda")
    scratch = torch.empty(B, M, device="cuda")
    rc = L.vdb_cmn_stem(feats.data_ptr(), fr.data_ptr(), B, t_max, M, 1, w.data_ptr(),
                        b.data_ptr(), OC, scratch.data_ptr(), y_ref.data_ptr(), None)
    assert rc == 0, vd.last_error()
    rc = L.vdb_cmn_stem_noalloc(feats.data_ptr(), fr.data_ptr(), B, t_max, M, 1, w.data_ptr(),
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


def test_noalloc_rejects_oversized_batch(cuda_lib):
    L = cuda_lib.lib()
    # 820 clips x 80 mels = 65600 means > 65536: rejected before any work
    rc = L.vdb_cmn_stem_noalloc(1, 1, 820, 10, 80, 1, 1, 1, 32, 1, None)
    assert rc != 0
    assert "65536" in cuda_lib.last_error()
