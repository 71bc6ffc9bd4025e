"""q8_0 weights kept as q8_0 on the device (int8 values + an f16 scale per 32 input
channels, expanded to f16 in the conv kernel's shared memory) against the same GGUF
with the q8_0 tensors widened to f16 on the host (VDB_Q8_WIDEN=1): bit-identical
embeddings, since both paths feed the tensor cores the same f16 values
f16(float(q) * float(d)). Parity of the q8_0 engine with the oracle on the dequantised
weights is covered by test_workload_gpu.py; this pins the device expansion."""
import os

import numpy as np
import pytest

import vd_synth

pytestmark = pytest.mark.gpu


def _embed(vd, path, clips, widen):
    old = os.environ.get("VDB_Q8_WIDEN")
    if widen:
        os.environ["VDB_Q8_WIDEN"] = "1"
    else:
        os.environ.pop("VDB_Q8_WIDEN", None)
    try:
        m = vd.Model(path)
    finally:
        if old is None:
            os.environ.pop("VDB_Q8_WIDEN", None)
        else:
            os.environ["VDB_Q8_WIDEN"] = old
    try:
        return m.embed_batch(clips), m.embed_batch(clips)
    finally:
        m.close()


def test_q8_device_expansion_equals_host_widening(tmp_path, cuda_lib):
    path = str(tmp_path / "r_q8.gguf")
    vd_synth.write_resnet_gguf(path, vd_synth.resnet34_model(21), "q8_0")
    lens = vd_synth.clip_lengths(5, 20, 2.0, 12.0)
    clips = [vd_synth.clip_f32(vd_synth.make_clip(300 + i, int(n))) for i, n in enumerate(lens)]
    dev_a, dev_b = _embed(cuda_lib, path, clips, widen=False)
    host_a, host_b = _embed(cuda_lib, path, clips, widen=True)
    assert np.array_equal(dev_a, host_a)
    assert np.array_equal(dev_b, host_b)  # graph-replayed call too


def test_q8_device_weights_are_about_half_the_f16_footprint(tmp_path, cuda_lib):
    """The ResNet34 block conv weights of a q8_0 GGUF: 1.0625 bytes per weight on the
    device (int8 + an f16 scale per 32) against 2 when widened to f16."""
    path = str(tmp_path / "r_q8.gguf")
    vd_synth.write_resnet_gguf(path, vd_synth.resnet34_model(21), "q8_0")
    sizes = {}
    for widen in (False, True):
        if widen:
            os.environ["VDB_Q8_WIDEN"] = "1"
        try:
            m = cuda_lib.Model(path)
        finally:
            os.environ.pop("VDB_Q8_WIDEN", None)
        sizes[widen] = m.conv_weight_bytes
        m.close()
    ratio = sizes[False] / sizes[True]
    assert abs(ratio - 1.0625 / 2) < 0.01, sizes
