"""Host-side layout helpers of vd_b200 (the GPU tests build their inputs with them):
GRID / PHASE / FPHASE / TPHASE / SEQ round trips on CPU tensors with ragged clip
lengths, and the plane / row formulas the header (include/vdb_ops.h) states for the
phase-split layouts. No GPU needed."""
import pytest

torch = pytest.importorskip("torch")
import vd_b200 as vd  # noqa: E402


def _ragged(B, C, F, T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, C, F, T, generator=g).half().float()
    tv = [T] + [max(1, T - 3 * b - 1) for b in range(1, B)]
    for b, t in enumerate(tv):
        x[b, ..., t:] = 0
    return x, tv


@pytest.mark.parametrize("F,T", [(80, 37), (41, 29), (10, 1)])
def test_grid_phase_fphase_round_trips(F, T):
    x, tv = _ragged(3, 16, F, T, F + T)
    assert torch.equal(vd.from_grid(vd.to_grid(x, tv), 3, 16, F, T), x)
    assert torch.equal(vd.from_phase(vd.to_phase(x, tv), 3, 16, F, T), x)
    assert torch.equal(vd.from_fphase(vd.to_fphase(x, tv), 3, 16, F, T), x)


def test_fphase_plane_formula():
    """Padded (tp, fp) of image b sits in plane fp&1 at row (b*(T+2)+tp)*(Fo+2)+(fp>>1)+1."""
    B, C, F, T = 2, 16, 9, 5
    x, tv = _ragged(B, C, F, T, 3)
    Fo = vd.out_extent(F, 2)
    fp_ = vd.to_fphase(x, tv)
    plane_rows = B * (T + 2) * (Fo + 2)
    for b in range(B):
        for t in range(T):
            for f in range(F):
                tp, fpp = t + 1, f + 1
                row = (fpp & 1) * plane_rows + (b * (T + 2) + tp) * (Fo + 2) + (fpp >> 1) + 1
                assert torch.equal(fp_[row].float(), x[b, :, f, t])


@pytest.mark.parametrize("T", [1, 2, 41, 200])
def test_tphase_round_trip_and_formula(T):
    """Frame u of clip b in plane u&1 at SEQ row b*(To+2P)+P+(u>>1); zero elsewhere."""
    g = torch.Generator().manual_seed(T)
    B, C, P = 3, 24, 2
    x = torch.randn(B, C, T, generator=g).half().float()
    tv = [T] + [max(1, T - 5 * b) for b in range(1, B)]
    for b, t in enumerate(tv):
        x[b, :, t:] = 0
    tp_ = vd.to_tphase(x, P, tv)
    To = vd.out_extent(T, 2)
    assert tp_.shape == (2 * B * (To + 2 * P), C)
    assert torch.equal(vd.from_tphase(tp_, B, C, T, P), x)
    rows = B * (To + 2 * P)
    written = torch.zeros(tp_.shape[0], dtype=torch.bool)
    for b, t in enumerate(tv):
        for u in range(t):
            r = (u & 1) * rows + b * (To + 2 * P) + P + (u >> 1)
            assert torch.equal(tp_[r].float(), x[b, :, u])
            written[r] = True
    assert torch.count_nonzero(tp_[~written]) == 0


def test_seq_zero_and_reflect_padding():
    g = torch.Generator().manual_seed(7)
    B, C, T, P = 2, 16, 9, 3
    x = torch.randn(B, C, T, generator=g).half().float()
    tv = [T, 6]
    z = vd.to_seq(x, P, tv, reflect=False).reshape(B, T + 2 * P, C)
    r = vd.to_seq(x, P, tv, reflect=True).reshape(B, T + 2 * P, C)
    for b, t in enumerate(tv):
        assert torch.equal(z[b, P:P + t].t().float(), x[b, :, :t])
        assert torch.count_nonzero(z[b, :P]) == 0 and torch.count_nonzero(z[b, P + t:]) == 0
        for j in range(1, P + 1):  # SpeechBrain reflect padding at the clip's own length
            assert torch.equal(r[b, P - j], r[b, P + j])
            assert torch.equal(r[b, P + t - 1 + j], r[b, P + t - 1 - j])
    assert torch.equal(vd.from_seq(z.reshape(-1, C), B, C, T, P)[1, :, :6], x[1, :, :6])


def test_qpack_round_trip_and_row_formula():
    """QPACK: row (b*(T+2) + t')*Wq + q holds padded pixels f' = 4q + j as channels
    j*32 .. j*32 + 31; a round trip returns the interior and every other slot is 0."""
    import torch
    import vd_b200 as vd
    B, F, T = 2, 18, 5
    x = torch.randn(B, 32, F, T)
    q = vd.to_qpack(x, [5, 3])
    Wq = vd.qpack_width(F)
    assert Wq == 5 and q.shape == (B * (T + 2) * Wq, 128)
    back = vd.from_qpack(q, B, F, T)
    want = x.half().float().clone()
    want[1, :, :, 3:] = 0
    assert torch.equal(back, want)
    b, t, f, c = 1, 2, 13, 7  # padded (t+1, f+1)
    row = (b * (T + 2) + t + 1) * Wq + (f + 1) // 4
    assert q[row, ((f + 1) % 4) * 32 + c] == x[b, c, f, t].half()
    full = vd.from_qpack(q, B, F, T, interior=False)
    mask = torch.zeros_like(full, dtype=torch.bool)
    mask[:, :, 1:F + 1, 1:T + 1] = True
    assert torch.all(full[~mask] == 0)
