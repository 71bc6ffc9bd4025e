"""Context lifecycle on the GPU: releasing the graph cache and workspace, freeing and
reloading a context, and two contexts side by side on one device.

Every comparison here is bit-exact. The engine's kernels reduce in a fixed order (no
floating-point atomics), so the same clips through the same weights give the same
bits whether the bucket ran eagerly, from a freshly captured CUDA graph, from a graph
captured before a cache release, or next to another context's work.
"""
import threading

import numpy as np
import pytest

import vd_synth

pytestmark = pytest.mark.gpu


def _clips(seed, n=24):
    lens = vd_synth.clip_lengths(seed, n, 2.0, 12.0)
    return [vd_synth.clip_f32(vd_synth.make_clip(seed * 100 + i, int(L)))
            for i, L in enumerate(lens)]


@pytest.fixture(scope="module")
def gguf_pair(tmp_path_factory):
    d = tmp_path_factory.mktemp("lifecycle")
    a = d / "resnet34_q8_0.gguf"
    b = d / "eres2net_f32.gguf"
    vd_synth.write_resnet_gguf(str(a), vd_synth.resnet34_model(11), "q8_0")
    vd_synth.write_eres2net_gguf(str(b), vd_synth.eres2net_model(12), "f32")
    return str(a), str(b)


def test_release_cache_then_reembed_is_bit_identical(cuda_lib, gguf_pair):
    clips = _clips(3)
    model = cuda_lib.Model(gguf_pair[0])
    try:
        # first call runs eagerly, the second captures the bucket graphs, the third
        # replays them
        runs = [model.embed_batch(clips) for _ in range(3)]
        model.release_cache()
        runs += [model.embed_batch(clips) for _ in range(3)]
        model.release_cache()
        model.release_cache()  # releasing an empty cache is a no-op
        runs.append(model.embed_batch(clips[:5]))
    finally:
        model.close()
    for r in runs[1:6]:
        assert np.array_equal(r, runs[0])
    assert np.array_equal(runs[6], runs[0][:5])


def test_free_and_reload_is_bit_identical(cuda_lib, gguf_pair):
    clips = _clips(4)
    outs = []
    for _ in range(3):
        model = cuda_lib.Model(gguf_pair[0])
        try:
            outs.append(model.embed_batch(clips))
            outs.append(model.embed_batch(clips))
        finally:
            model.close()
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_two_contexts_side_by_side(cuda_lib, gguf_pair):
    """A ResNet34 and an ERes2Net context on the same device: interleaved calls and
    calls from two host threads at once each equal the context's solo result."""
    ca, cb = _clips(5), _clips(6, 17)
    solo = []
    for path, clips in zip(gguf_pair, (ca, cb)):
        m = cuda_lib.Model(path)
        try:
            solo.append(m.embed_batch(clips))
        finally:
            m.close()
    ma, mb = cuda_lib.Model(gguf_pair[0]), cuda_lib.Model(gguf_pair[1])
    try:
        for _ in range(2):
            assert np.array_equal(ma.embed_batch(ca), solo[0])
            assert np.array_equal(mb.embed_batch(cb), solo[1])
        res = {}
        errs = []

        def worker(name, m, clips):
            try:
                res[name] = [m.embed_batch(clips) for _ in range(4)]
            except Exception as e:  # reported on the main thread
                errs.append(e)

        ts = [threading.Thread(target=worker, args=("a", ma, ca)),
              threading.Thread(target=worker, args=("b", mb, cb))]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=300)
        assert not errs, errs
        assert all(np.array_equal(r, solo[0]) for r in res["a"])
        assert all(np.array_equal(r, solo[1]) for r in res["b"])
        # releasing one context's cache leaves the other's untouched
        ma.release_cache()
        assert np.array_equal(mb.embed_batch(cb), solo[1])
        assert np.array_equal(ma.embed_batch(ca), solo[0])
    finally:
        ma.close()
        mb.close()
