"""Image preprocessing without a GPU: the oracle against the reference's four
media known-answer tests (src/media/mod.rs:1336-1464), and the C ABI's
validation messages (src/media/mod.rs:185-193, 224-241, 296-311, 384-398,
492-509)."""
import ctypes as C

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O


def test_packed_rgb_to_nchw_known_answer():
    # src/media/mod.rs:1339-1375
    frame = np.array([255, 0, 0, 0, 255, 0, 0, 0, 255, 255, 255, 255], np.uint8).reshape(1, 2, 2, 3)
    out = O.preprocess_packed(frame, 0, 2, 2).ravel()
    expected = [1, 0, 0, 1, 0, 1, 0, 1, 0, 0, 1, 1]
    assert np.abs(out - expected).max() <= 1e-6


def test_packed_bgr_into_history_slot_known_answer():
    # src/media/mod.rs:1377-1402
    frame = np.array([0, 128, 255], np.uint8).reshape(1, 1, 1, 3)
    out = O.preprocess_packed(frame, 1, 1, 1, history_len=3, slot=1).ravel()
    expected = [0, 0, 0, 1, 128 / 255, 0, 0, 0, 0]
    assert np.abs(out - expected).max() <= 1e-6


def test_nv12_to_nchw_known_answer():
    # src/media/mod.rs:1404-1429
    y = np.zeros((1, 2, 2), np.uint8)
    uv = np.full((1, 1, 1, 2), 128, np.uint8)
    out = O.preprocess_nv12(y, uv, 2, 2, 2)
    assert out.size == 12 and np.abs(out).max() <= 1e-6


def test_nv12_into_history_slot_known_answer():
    # src/media/mod.rs:1431-1463
    y = np.full((1, 2, 2), 255, np.uint8)
    uv = np.full((1, 1, 1, 2), 128, np.uint8)
    out = O.preprocess_nv12(y, uv, 3, 2, 2, history_len=2, slot=1).ravel()
    assert out.size == 24
    assert np.abs(out[:12]).max() <= 1e-6
    assert np.abs(out[12:] - 1.0).max() <= 1e-6


def test_imagenet_224_preset():
    # ImagePreprocess::imagenet_224 (src/media/mod.rs:175-183)
    c = L.ImagePreprocess.imagenet_224()
    assert (c.output_height, c.output_width) == (224, 224)
    np.testing.assert_array_equal(np.array(c.mean), np.float32([0.485, 0.456, 0.406]))
    np.testing.assert_array_equal(np.array(c.std), np.float32([0.229, 0.224, 0.225]))


def _packed(cfg, B=1, H=2, W=2, fmt=0, history_len=0, slot=0):
    status = L.lib.lwm_preprocess_packed_device(None, None, B, H, W, fmt, C.byref(cfg), history_len, slot, 0, None)
    return status, L.lib.lwm_last_error().decode()


def _nv12(cfg, B=1, H=2, W=2, cs=0, history_len=0, slot=0):
    status = L.lib.lwm_preprocess_nv12_device(None, None, None, B, H, W, cs, C.byref(cfg), history_len, slot, 0,
                                              None)
    return status, L.lib.lwm_last_error().decode()


@pytest.mark.parametrize("call, message", [
    (lambda c: _packed(c, H=0), "packed CUDA image dimensions must be greater than zero"),
    (lambda c: _packed(c, B=0), "packed CUDA image dimensions must be greater than zero"),
    (lambda c: _nv12(c, W=0), "NV12 CUDA image dimensions must be greater than zero"),
    (lambda c: _nv12(c, H=3, W=4), "NV12 CUDA image dimensions must be even, got 3x4"),
    (lambda c: _packed(c, history_len=3, slot=3), "CUDA image history slot 3 is outside history_len 3"),
    (lambda c: _nv12(c, history_len=2, slot=5), "CUDA NV12 history slot 5 is outside history_len 2"),
    (lambda c: _packed(c, fmt=4), "unknown packed image format 4; expected 0=RGB, 1=BGR, 2=RGBA, or 3=BGRA"),
])
def test_preprocess_validation_messages(call, message):
    status, msg = call(L.ImagePreprocess.make(2, 2))
    assert status == 1 and msg == message


def test_preprocess_config_validation_messages():
    status, msg = _packed(L.ImagePreprocess.make(0, 2))
    assert status == 1 and msg == "CUDA preprocess output dimensions must be greater than zero"
    status, msg = _nv12(L.ImagePreprocess.make(2, 2, std=(1.0, 0.0, 1.0)))
    assert status == 1 and msg == "CUDA preprocess std values must be non-zero"
    # a valid request without a context reaches the null check
    status, msg = _packed(L.ImagePreprocess.make(2, 2))
    assert status == 1 and msg == "null argument"


def test_oracle_resize_is_bilinear_with_half_pixel_centres():
    # 2x upscaling of a ramp: samples sit at quarter positions, edges clamp
    frame = np.zeros((1, 1, 4, 3), np.uint8)
    frame[0, 0, :, 0] = [0, 40, 80, 120]
    out = O.preprocess_packed(frame, 0, 1, 8)[0, 0, 0] * 255
    np.testing.assert_allclose(out, [0, 10, 30, 50, 70, 90, 110, 120], atol=1e-4)
