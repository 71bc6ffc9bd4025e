"""Generate the committed golden fixtures in tests/golden/ (run where the
reference checkout and torchaudio are available; the fixtures then travel with
the repository).

* fbank_torchaudio.npz -- three seeded synthetic clips (int16) and their
  torchaudio.compliance.kaldi.fbank features with the reference's options
  (povey window, preemph 0.97, dither 0, snip_edges, 80 mels) and per-utterance
  CMN: the same golden source the reference's own parity suite uses
  (scripts/gen_baseline.py:73-81 in the reference).
* ref_conv_kat.npz -- outputs of the reference's OWN blocked conv kernels
  (oracle/_ref/libvdref.so, src/directconv.cpp compiled unmodified) on the
  shapes of the reference's tests/test_blocked.cpp:107-109,137-138,168-169, with
  seeded U(-1, 1) inputs.
* ref_resnet_tiny.npz -- pre-norm and L2 embeddings of a small seeded ResNet
  (vd_synth.tiny_resnet_model) from the reference kernels + restated glue.
* ref_eres2net_tiny.npz -- the same for a small seeded ERes2Net
  (vd_synth.tiny_eres2net_model: every block kind, AFF and cross-stage fusion).
* ref_ecapa_tiny.npz -- a small seeded ECAPA-TDNN (vd_synth.tiny_ecapa_model) on
  two clips: torchaudio FBank features and the float64 torch forward
  (vd_synth.ecapa_forward_torch: torch's reflect pad, conv1d, batch_norm,
  softmax), independent of the numpy oracle it pins. The reference's own ECAPA
  graph needs the absent ggml library, so no reference output exists for it.
* ref_campplus_tiny.npz -- the same for a small seeded CAM++ (vd_synth.tiny_campplus_model,
  every layer kind; one clip longer than one 100-frame context segment) from
  vd_synth.campplus_forward_torch.
* fixtures_ref.npz -- the reference's real-audio fixtures (fixtures/*.wav, copied
  from its tests/fixtures): per clip the reference's own decode + resample
  (vd::load_audio_16k_mono, src/audio_io.cpp:25-38, compiled into oracle/_ref), the
  reference's own post-CMN FBank of those samples (src/fbank.cpp compiled) and
  torchaudio's Kaldi FBank of the same samples.

Usage: python tests/golden/make_golden.py [name ...]   (default: every fixture)
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "voice-detect.cpp_b200"))

import oracle  # noqa: E402
import vd_synth  # noqa: E402

CONV_KAT = [
    # (W=time, H=freq, IC, OC, stride, bias_relu, k)
    (20, 11, 32, 64, 1, False, 3),
    (20, 11, 64, 128, 2, False, 3),
    (7, 5, 16, 16, 1, False, 3),
    (20, 11, 32, 64, 1, True, 3),
    (20, 11, 64, 128, 2, True, 3),
    (20, 11, 64, 128, 2, False, 1),
    (15, 9, 32, 64, 2, False, 1),
]


def fbank_torchaudio(pcm: np.ndarray) -> np.ndarray:
    import torch
    import torchaudio
    x = torch.from_numpy(pcm.astype(np.float64))[None]
    f = torchaudio.compliance.kaldi.fbank(x, num_mel_bins=80, frame_length=25, frame_shift=10,
                                          dither=0.0, window_type="povey", preemphasis_coefficient=0.97,
                                          remove_dc_offset=True, snip_edges=True,
                                          sample_frequency=16000, low_freq=20.0, high_freq=0.0,
                                          energy_floor=0.0, use_energy=False)
    f = f - f.mean(0, keepdim=True)
    return f.numpy().T.astype(np.float32)  # [80, T]


def conv_inputs(i: int, W, H, IC, OC, k):
    rng = np.random.default_rng(1234 + i)
    x = rng.uniform(-1, 1, (IC, H, W)).astype(np.float32)
    w = rng.uniform(-1, 1, (OC, IC, k, k)).astype(np.float32)
    b = rng.uniform(-1, 1, OC).astype(np.float32)
    return x, w, b


def make_ecapa() -> None:
    import torch
    m = vd_synth.tiny_ecapa_model(7, n_mels=80)
    d = {}
    for i, (seed, n) in enumerate(((23, 28000), (24, 16000 + 160 * 9 + 55))):
        pcm = vd_synth.clip_f32(vd_synth.make_clip(seed, n))
        feats = fbank_torchaudio(pcm)
        emb, pre = vd_synth.ecapa_forward_torch(m, torch.from_numpy(feats[None].astype(np.float64)))
        d[f"pcm{i}"] = pcm
        d[f"feats{i}"] = feats
        d[f"emb{i}"] = emb[0].astype(np.float32)
        d[f"prenorm{i}"] = pre[0].astype(np.float32)
    np.savez_compressed(HERE / "ref_ecapa_tiny.npz", **d)


def make_campplus() -> None:
    import torch
    m = vd_synth.tiny_campplus_model(9, n_mels=80)
    d = {}
    for i, (seed, n) in enumerate(((25, 24000), (26, 16000 + 160 * 230 + 61))):
        pcm = vd_synth.clip_f32(vd_synth.make_clip(seed, n))
        feats = fbank_torchaudio(pcm)
        emb, pre = vd_synth.campplus_forward_torch(m, torch.from_numpy(feats[None].astype(np.float64)))
        d[f"pcm{i}"] = pcm
        d[f"feats{i}"] = feats
        d[f"emb{i}"] = emb[0].astype(np.float32)
        d[f"prenorm{i}"] = pre[0].astype(np.float32)
    np.savez_compressed(HERE / "ref_campplus_tiny.npz", **d)


FIXTURES = ("clip_a", "clip_b_same", "clip_c_diff")


def make_fixtures() -> None:
    d = {}
    for name in FIXTURES:
        pcm = oracle.ref_load_audio_16k_mono(HERE / "fixtures" / f"{name}.wav")
        d[f"{name}_pcm"] = pcm
        d[f"{name}_ref_fbank"] = oracle.ref_fbank(pcm)
        d[f"{name}_ta_fbank"] = fbank_torchaudio(pcm)
    np.savez_compressed(HERE / "fixtures_ref.npz", **d)


def main() -> None:
    if len(sys.argv) > 1:
        for name in sys.argv[1:]:
            {"ecapa": make_ecapa, "campplus": make_campplus, "fixtures": make_fixtures}[name]()
        print("wrote", sys.argv[1:])
        return
    clips = [vd_synth.make_clip(s, n) for s, n in ((11, 48000), (12, 16000 + 37), (13, 401))]
    d = {}
    for i, c in enumerate(clips):
        d[f"clip{i}"] = c
        d[f"fbank{i}"] = fbank_torchaudio(vd_synth.clip_f32(c))
    np.savez_compressed(HERE / "fbank_torchaudio.npz", **d)

    d = {}
    for i, (W, H, IC, OC, s, br, k) in enumerate(CONV_KAT):
        x, w, b = conv_inputs(i, W, H, IC, OC, k)
        if k == 3:
            y = oracle.ref_conv3x3(x, w, s, b if br else None, br)
        else:
            y = oracle.ref_conv1x1(x, w, s)
        d[f"y{i}"] = y
    np.savez_compressed(HERE / "ref_conv_kat.npz", **d)

    m = vd_synth.tiny_resnet_model(5, n_mels=80)
    pcm = vd_synth.clip_f32(vd_synth.make_clip(21, 24000))
    feats = oracle.ref_fbank(pcm)
    R = oracle.RefResNet34(m)
    emb, pre = R.embed(feats)
    np.savez_compressed(HERE / "ref_resnet_tiny.npz", pcm=pcm, emb=emb, prenorm=pre)

    m = vd_synth.tiny_eres2net_model(6, n_mels=80)
    pcm = vd_synth.clip_f32(vd_synth.make_clip(22, 20000))
    feats = oracle.ref_fbank(pcm)
    emb, pre = oracle.RefERes2Net(m).embed(feats)
    np.savez_compressed(HERE / "ref_eres2net_tiny.npz", pcm=pcm, emb=emb, prenorm=pre)
    make_ecapa()
    make_campplus()
    make_fixtures()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
