"""The audio front door, pinned bitwise to the reference's own code (no GPU needed).

The reference decodes WAV files with its vendored dr_wav, averages channels in f64
and resamples linearly to 16 kHz (vd::load_audio_16k_mono / vd::resample_linear,
src/audio_io.cpp:9-38). oracle/_ref compiles that file unmodified; these tests hold
the product's own WAV reader and resampler (csrc/audio.cpp, reached through
voicedetect_b200_load_audio_16k_mono, the decode that embed_path and verify_paths
use) and the oracle's C restatement to it, bit for bit, over every encoding the
reader accepts, several channel counts and sample rates, and the reference's
real-audio fixtures.
"""
import struct
from pathlib import Path

import numpy as np
import pytest

import oracle
import vd_b200

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = ("clip_a", "clip_b_same", "clip_c_diff")

needs_ref = pytest.mark.skipif(not oracle.ref_available(),
                               reason="oracle/_ref (the reference compiled) not built")


def _write_wav(path, samples: np.ndarray, sr: int, fmt: str, extensible: bool = False):
    """samples: [frames, channels] float64 in [-1, 1). fmt: u8 s16 s24 s32 f32 f64."""
    frames, ch = samples.shape
    x = samples.reshape(-1)
    if fmt == "u8":
        data, tag, bits = np.clip(np.round(x * 128 + 128), 0, 255).astype(np.uint8).tobytes(), 1, 8
    elif fmt == "s16":
        data, tag, bits = np.clip(np.round(x * 32768), -32768, 32767).astype("<i2").tobytes(), 1, 16
    elif fmt == "s24":
        v = np.clip(np.round(x * 8388608), -8388608, 8388607).astype(np.int64) & 0xFFFFFF
        b = np.stack([v & 0xFF, (v >> 8) & 0xFF, (v >> 16) & 0xFF], 1).astype(np.uint8)
        data, tag, bits = b.tobytes(), 1, 24
    elif fmt == "s32":
        data, tag, bits = (np.clip(np.round(x * 2147483648.0), -2147483648, 2147483647)
                           .astype("<i4").tobytes(), 1, 32)
    elif fmt == "f32":
        data, tag, bits = x.astype("<f4").tobytes(), 3, 32
    elif fmt == "f64":
        data, tag, bits = x.astype("<f8").tobytes(), 3, 64
    else:
        raise ValueError(fmt)
    block = ch * bits // 8
    if extensible:
        guid = struct.pack("<IHH8s", tag, 0x0000, 0x0010, b"\x80\x00\x00\xaa\x00\x38\x9b\x71")
        fmt_body = struct.pack("<HHIIHHHHI", 0xFFFE, ch, sr, sr * block, block, bits, 22, bits,
                               0) + guid
    else:
        fmt_body = struct.pack("<HHIIHH", tag, ch, sr, sr * block, block, bits)
    body = b"WAVE" + b"fmt " + struct.pack("<I", len(fmt_body)) + fmt_body
    body += b"data" + struct.pack("<I", len(data)) + data + (b"\0" if len(data) & 1 else b"")
    Path(path).write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)


def _signal(seed: int, frames: int, ch: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    t = np.arange(frames)[:, None]
    x = 0.5 * np.sin(2 * np.pi * (t * (0.01 + 0.003 * np.arange(ch))) + rng.uniform(0, 6, ch))
    x += 0.2 * rng.standard_normal((frames, ch))
    return np.clip(x, -0.999, 0.999)


@needs_ref
@pytest.mark.parametrize("fmt", ["u8", "s16", "s24", "s32", "f32", "f64"])
@pytest.mark.parametrize("ch", [1, 2, 3])
def test_wav_decode_matches_reference_bitwise(tmp_path, fmt, ch):
    """16 kHz files (no resampling): the decode and channel average alone."""
    p = tmp_path / f"x_{fmt}_{ch}.wav"
    _write_wav(p, _signal(len(fmt) * 7 + ch, 4001, ch), 16000, fmt)
    want = oracle.ref_load_audio_16k_mono(p)
    got = vd_b200.load_audio_16k_mono(p)
    assert got.dtype == np.float32 and len(got) == len(want) == 4001
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{fmt}/{ch}ch: {np.count_nonzero(got != want)} samples differ"


@needs_ref
@pytest.mark.parametrize("fmt", ["s16", "f32"])
def test_wav_extensible_format_matches_reference(tmp_path, fmt):
    p = tmp_path / f"ext_{fmt}.wav"
    _write_wav(p, _signal(3, 1500, 2), 16000, fmt, extensible=True)
    want = oracle.ref_load_audio_16k_mono(p)
    got = vd_b200.load_audio_16k_mono(p)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("sr", [8000, 11025, 22050, 24000, 44100, 48000])
@pytest.mark.parametrize("fmt,ch", [("s16", 1), ("s24", 2), ("f32", 1)])
def test_load_and_resample_matches_reference_bitwise(tmp_path, sr, fmt, ch):
    """Decode + f64 downmix + linear resample to 16 kHz, end to end."""
    p = tmp_path / f"r_{sr}_{fmt}.wav"
    _write_wav(p, _signal(sr + ch, sr // 3 + 17, ch), sr, fmt)
    want = oracle.ref_load_audio_16k_mono(p)
    got = vd_b200.load_audio_16k_mono(p)
    assert len(got) == len(want)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("sr", [8000, 22050, 44100, 48000, 16001, 96000])
def test_oracle_resample_matches_reference_bitwise(sr):
    """The oracle's C restatement of resample_linear (the checker the device ingest
    tests use) against the reference's compiled function, including the
    one-sample and empty edge cases."""
    rng = np.random.default_rng(sr)
    for n in (0, 1, 2, 3, 997, sr + 5):
        x = rng.uniform(-1, 1, n).astype(np.float32)
        want = oracle.ref_resample_linear(x, sr, 16000)
        got = oracle.resample_linear(x, sr, 16000)
        assert len(got) == len(want), (n, len(got), len(want))
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), n


@needs_ref
@pytest.mark.parametrize("name", FIXTURES)
def test_reference_fixture_decode_matches_bitwise(name):
    """The reference's own real-audio fixtures: the product decode equals the
    reference's, and both equal the committed golden samples."""
    p = GOLDEN / "fixtures" / f"{name}.wav"
    want = oracle.ref_load_audio_16k_mono(p)
    got = vd_b200.load_audio_16k_mono(p)
    gold = np.load(GOLDEN / "fixtures_ref.npz")[f"{name}_pcm"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(gold.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_fbank_oracle_matches_reference(name):
    """Real-audio FBank, with the reference's own gate (tests/test_fbank.cpp:56-59:
    max|d| <= 1e-3 and cosine >= 0.9999): the C restatement against the reference's
    compiled fbank.cpp (committed golden) and against torchaudio's Kaldi FBank."""
    d = np.load(GOLDEN / "fixtures_ref.npz")
    pcm = d[f"{name}_pcm"]
    got = oracle.fbank(pcm)
    for key in ("ref_fbank", "ta_fbank"):
        want = d[f"{name}_{key}"]
        assert got.shape == want.shape == (80, 298)
        cos = float((got.astype(np.float64) * want).sum() /
                    (np.linalg.norm(got) * np.linalg.norm(want)))
        assert np.abs(got - want).max() <= 1e-3 and cos >= 0.9999, (key, cos)
    # the restatement is bit-exact to the compiled reference
    assert np.array_equal(got, d[f"{name}_ref_fbank"])


def test_load_audio_rejects_bad_files(tmp_path):
    bad = tmp_path / "bad.wav"
    bad.write_bytes(b"RIFF\x04\x00\x00\x00WAVE")
    for p in (bad, tmp_path / "missing.wav", tmp_path):
        with pytest.raises(RuntimeError):
            vd_b200.load_audio_16k_mono(p)
