"""Image preprocessing on the GPU through the C ABI against the oracle
(swm_packed_u8_to_nchw_f32 / swm_nv12_to_nchw_f32, src/media/mod.rs:1113-1333).

The kernels are built with -fmad=false and IEEE division, and the oracle with
-ffp-contract=off, so f32 outputs are expected bit-identical; bf16 outputs are
the oracle's f32 values rounded to nearest-even."""
import zlib

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

IMAGENET = dict(mean=(0.485, 0.456, 0.406), std=(0.229, 0.224, 0.225))


def _bf16_of(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(x).to(torch.bfloat16).float().numpy()


def _run_packed(ctx, frames, fmt, oh, ow, history_len=0, slot=0, bf16=False, **norm):
    B, H, W, _ = frames.shape
    cfg = L.ImagePreprocess.make(oh, ow, **norm) if norm else L.ImagePreprocess.make(oh, ow)
    dev = torch.from_numpy(frames).cuda()
    shape = (B, 3, oh, ow) if history_len == 0 else (B, history_len, 3, oh, ow)
    out = torch.full(shape, 7.0, device="cuda", dtype=torch.bfloat16 if bf16 else torch.float32)
    torch.cuda.synchronize()
    L.preprocess_packed_device(ctx, dev, B, H, W, fmt, cfg, out, history_len, slot, bf16)
    ctx.synchronize()
    return out.float().cpu().numpy()


def _run_nv12(ctx, y, uv, cs, oh, ow, history_len=0, slot=0, bf16=False, **norm):
    B, H, W = y.shape
    cfg = L.ImagePreprocess.make(oh, ow, **norm) if norm else L.ImagePreprocess.make(oh, ow)
    shape = (B, 3, oh, ow) if history_len == 0 else (B, history_len, 3, oh, ow)
    out = torch.full(shape, 7.0, device="cuda", dtype=torch.bfloat16 if bf16 else torch.float32)
    torch.cuda.synchronize()
    L.preprocess_nv12_device(ctx, torch.from_numpy(y).cuda(), torch.from_numpy(uv).cuda(), B, H, W, cs, cfg, out,
                             history_len, slot, bf16)
    ctx.synchronize()
    return out.float().cpu().numpy()


def test_reference_known_answers_on_gpu(ctx):
    # the four tests of src/media/mod.rs:1336-1464, on the CUDA path
    rgb = np.array([255, 0, 0, 0, 255, 0, 0, 0, 255, 255, 255, 255], np.uint8).reshape(1, 2, 2, 3)
    got = _run_packed(ctx, rgb, "rgb", 2, 2).ravel()
    assert np.abs(got - [1, 0, 0, 1, 0, 1, 0, 1, 0, 0, 1, 1]).max() <= 1e-6
    bgr = np.array([0, 128, 255], np.uint8).reshape(1, 1, 1, 3)
    got = _run_packed(ctx, bgr, "bgr", 1, 1, history_len=3, slot=1).ravel()
    want = np.array([7, 7, 7, 1, 128 / 255, 0, 7, 7, 7])  # other slots untouched
    assert np.abs(got - want).max() <= 1e-6
    y0 = np.zeros((1, 2, 2), np.uint8)
    uv = np.full((1, 1, 1, 2), 128, np.uint8)
    assert np.abs(_run_nv12(ctx, y0, uv, "bt601-full", 2, 2)).max() <= 1e-6
    y1 = np.full((1, 2, 2), 255, np.uint8)
    got = _run_nv12(ctx, y1, uv, "bt709-full", 2, 2, history_len=2, slot=1).ravel()
    assert np.abs(got[12:] - 1.0).max() <= 1e-6 and (got[:12] == 7.0).all()


@pytest.mark.parametrize("fmt", ["rgb", "bgr", "rgba", "bgra"])
@pytest.mark.parametrize("size", [(3, 480, 640, 224, 224), (2, 7, 5, 16, 12), (1, 1, 1, 3, 2), (2, 333, 517, 224, 224)])
def test_packed_matches_oracle_bit_exact(ctx, fmt, size):
    B, H, W, oh, ow = size
    rng = np.random.default_rng(zlib.crc32(repr((fmt, size)).encode()))
    frames = rng.integers(0, 256, (B, H, W, 4 if fmt.endswith("a") else 3), dtype=np.uint8)
    got = _run_packed(ctx, frames, fmt, oh, ow, **IMAGENET)
    ref = O.preprocess_packed(frames, L.PACKED_FORMATS[fmt], oh, ow, **IMAGENET)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("cs", ["bt601-video", "bt709-video", "bt601-full", "bt709-full"])
@pytest.mark.parametrize("size", [(2, 720, 1280, 224, 224), (1, 4, 6, 9, 7), (3, 2, 2, 1, 1)])
def test_nv12_matches_oracle_bit_exact(ctx, cs, size):
    B, H, W, oh, ow = size
    rng = np.random.default_rng(zlib.crc32(repr((cs, size)).encode()))
    y = rng.integers(0, 256, (B, H, W), dtype=np.uint8)
    uv = rng.integers(0, 256, (B, H // 2, W // 2, 2), dtype=np.uint8)
    got = _run_nv12(ctx, y, uv, cs, oh, ow, **IMAGENET)
    ref = O.preprocess_nv12(y, uv, L.NV12_COLOR_SPACES[cs], oh, ow, **IMAGENET)
    np.testing.assert_array_equal(got, ref)


def test_history_slots_fill_independently(ctx):
    rng = np.random.default_rng(5)
    B, H, W, hist = 2, 96, 128, 4
    out_ref = np.zeros((B, hist, 3, 64, 64), np.float32)
    cfg = L.ImagePreprocess.make(64, 64, **IMAGENET)
    out = torch.zeros((B, hist, 3, 64, 64), device="cuda")
    for slot in (2, 0, 3, 1):
        frames = rng.integers(0, 256, (B, H, W, 3), dtype=np.uint8)
        torch.cuda.synchronize()
        L.preprocess_packed_device(ctx, torch.from_numpy(frames).cuda(), B, H, W, "rgb", cfg, out, hist, slot)
        O.preprocess_packed(frames, 0, 64, 64, history_len=hist, slot=slot, out=out_ref, **IMAGENET)
    ctx.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), out_ref)


def test_bf16_output_is_rounded_oracle(ctx):
    rng = np.random.default_rng(9)
    frames = rng.integers(0, 256, (2, 300, 400, 3), dtype=np.uint8)
    got = _run_packed(ctx, frames, "rgb", 224, 224, bf16=True, **IMAGENET)
    ref = O.preprocess_packed(frames, 0, 224, 224, **IMAGENET)
    np.testing.assert_array_equal(got, _bf16_of(ref))
    y = rng.integers(0, 256, (2, 360, 640), dtype=np.uint8)
    uv = rng.integers(0, 256, (2, 180, 320, 2), dtype=np.uint8)
    got = _run_nv12(ctx, y, uv, "bt709-video", 224, 224, history_len=3, slot=2, bf16=True, **IMAGENET)
    ref = O.preprocess_nv12(y, uv, 1, 224, 224, **IMAGENET)
    np.testing.assert_array_equal(got[:, 2], _bf16_of(ref))
    assert (got[:, :2] == 7.0).all()


# Shapes the row-staged NV12 kernel takes (row bytes a multiple of 16, output
# width a multiple of 4): full HD at its own size, up- and down-scaling, the
# 4096-byte row buffers, and two-row frames (a single chroma row).
STAGED = [(1, 1080, 1920, 1080, 1920), (2, 64, 96, 200, 300), (1, 8, 4096, 16, 2048), (2, 720, 1280, 360, 640),
          (2, 2, 16, 1, 4), (1, 2, 16, 3, 8)]


@pytest.mark.parametrize("cs", ["bt601-video", "bt709-video", "bt601-full", "bt709-full"])
@pytest.mark.parametrize("size", STAGED)
def test_nv12_row_staged_matches_oracle_bit_exact(ctx, cs, size):
    B, H, W, oh, ow = size
    rng = np.random.default_rng(zlib.crc32(repr(("staged", cs, size)).encode()))
    y = rng.integers(0, 256, (B, H, W), dtype=np.uint8)
    uv = rng.integers(0, 256, (B, H // 2, W // 2, 2), dtype=np.uint8)
    got = _run_nv12(ctx, y, uv, cs, oh, ow, **IMAGENET)
    ref = O.preprocess_nv12(y, uv, L.NV12_COLOR_SPACES[cs], oh, ow, **IMAGENET)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("norm", [dict(mean=(0.0, 0.0, 0.0), std=(1.0, 1.0, 1.0)),
                                  dict(mean=(0.5, 0.01, 0.9), std=(0.01, 3.7, 1e-3)),
                                  dict(mean=(2.0 ** -40, -1000.0, 0.25), std=(2.0 ** -40, 2.0 ** 40, 0.3))])
def test_nv12_row_staged_division_is_exact(ctx, norm):
    # the staged kernel divides by std through a host reciprocal and two
    # remainder corrections; its quotients equal the oracle's IEEE division
    rng = np.random.default_rng(17)
    y = rng.integers(0, 256, (2, 360, 640), dtype=np.uint8)
    uv = rng.integers(0, 256, (2, 180, 320, 2), dtype=np.uint8)
    for cs in ("bt601-video", "bt709-full"):
        got = _run_nv12(ctx, y, uv, cs, 360, 640, **norm)
        ref = O.preprocess_nv12(y, uv, L.NV12_COLOR_SPACES[cs], 360, 640, **norm)
        np.testing.assert_array_equal(got, ref)


def test_nv12_staged_and_generic_kernels_agree(ctx):
    # an output that starts 4 bytes past a 16-byte boundary takes the generic
    # per-pixel kernel; both kernels write identical values
    rng = np.random.default_rng(23)
    B, H, W, oh, ow = 2, 480, 640, 240, 320
    y = torch.from_numpy(rng.integers(0, 256, (B, H, W), dtype=np.uint8)).cuda()
    uv = torch.from_numpy(rng.integers(0, 256, (B, H // 2, W // 2, 2), dtype=np.uint8)).cuda()
    cfg = L.ImagePreprocess.make(oh, ow, **IMAGENET)
    n = B * 3 * oh * ow
    aligned = torch.full((n,), 7.0, device="cuda")
    shifted = torch.full((n + 1,), 7.0, device="cuda")
    torch.cuda.synchronize()
    for out in (aligned, shifted[1:]):
        L.preprocess_nv12_device(ctx, y, uv, B, H, W, "bt601-video", cfg, out)
    ctx.synchronize()
    assert shifted[1:].data_ptr() % 16 == 4
    np.testing.assert_array_equal(aligned.cpu().numpy(), shifted[1:].cpu().numpy())
    assert float(shifted[0]) == 7.0


# Shapes the row-staged packed kernel takes (row bytes W x channels a multiple
# of 16 up to 8192, output width a multiple of 4): full HD at its own size
# (RGB 5760-byte and RGBA 7680-byte rows), up- and down-scaling, 2048-pixel
# RGBA rows, two-row frames.
PACKED_STAGED = [(1, 1080, 1920, 1080, 1920), (2, 32, 64, 100, 200), (2, 720, 1280, 360, 640),
                 (1, 4, 2048, 8, 2048), (1, 2, 16, 3, 8)]


@pytest.mark.parametrize("fmt", ["rgb", "bgr", "rgba", "bgra"])
@pytest.mark.parametrize("size", PACKED_STAGED)
def test_packed_row_staged_matches_oracle_bit_exact(ctx, fmt, size):
    B, H, W, oh, ow = size
    C = 4 if fmt in ("rgba", "bgra") else 3
    rng = np.random.default_rng(zlib.crc32(repr(("packed-staged", fmt, size)).encode()))
    frames = rng.integers(0, 256, (B, H, W, C), dtype=np.uint8)
    got = _run_packed(ctx, frames, fmt, oh, ow, **IMAGENET)
    ref = O.preprocess_packed(frames, L.PACKED_FORMATS[fmt], oh, ow, **IMAGENET)
    np.testing.assert_array_equal(got, ref)


def test_packed_staged_and_generic_kernels_agree(ctx):
    rng = np.random.default_rng(29)
    B, H, W, oh, ow = 2, 240, 320, 120, 160
    frames = torch.from_numpy(rng.integers(0, 256, (B, H, W, 3), dtype=np.uint8)).cuda()
    cfg = L.ImagePreprocess.make(oh, ow, mean=(0.5, 0.01, 0.9), std=(0.01, 3.7, 1e-3))
    n = B * 3 * oh * ow
    aligned = torch.full((n,), 7.0, device="cuda")
    shifted = torch.full((n + 1,), 7.0, device="cuda")
    torch.cuda.synchronize()
    for out in (aligned, shifted[1:]):
        L.preprocess_packed_device(ctx, frames, B, H, W, "rgb", cfg, out)
    ctx.synchronize()
    np.testing.assert_array_equal(aligned.cpu().numpy(), shifted[1:].cpu().numpy())


# ------------------------------------------------- ViT patch-matrix output

def _patchify(nchw: np.ndarray, p: int) -> np.ndarray:
    """[B, 3, H, W] -> [B, (H/p)(W/p), 3 p p]: the stride-p patch-embedding
    input (Embeddings, src/models/lewm/vit.rs:32-52)."""
    B, C, H, W = nchw.shape
    x = nchw.reshape(B, C, H // p, p, W // p, p).transpose(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // p) * (W // p), C * p * p)


# (B, H, W, oh, ow, p): row-staged shapes (widths multiple of 16, p multiple
# of 4) and per-pixel ones (odd source width, p = 2 is not a multiple of 4)
@pytest.mark.parametrize("shape", [(2, 480, 640, 224, 224, 16), (3, 224, 224, 224, 224, 16),
                                   (2, 90, 122, 32, 48, 8), (1, 64, 80, 12, 10, 2)])
@pytest.mark.parametrize("bf16", [False, True])
def test_nv12_patch_layout_equals_oracle_patchified(ctx, shape, bf16):
    B, H, W, oh, ow, p = shape
    rng = np.random.default_rng(zlib.crc32(repr(("nv12p", shape)).encode()))
    y = rng.integers(0, 256, (B, H, W), dtype=np.uint8)
    uv = rng.integers(0, 256, (B, H // 2, W // 2, 2), dtype=np.uint8)
    cfg = L.ImagePreprocess.make(oh, ow, **IMAGENET)
    out = torch.full((B, (oh // p) * (ow // p), 3 * p * p), 7.0, device="cuda",
                     dtype=torch.bfloat16 if bf16 else torch.float32)
    torch.cuda.synchronize()
    L.preprocess_nv12_patches_device(ctx, torch.from_numpy(y).cuda(), torch.from_numpy(uv).cuda(), B, H, W,
                                     "bt709-video", cfg, p, out, bf16)
    ctx.synchronize()
    ref = _patchify(O.preprocess_nv12(y, uv, 1, oh, ow, **IMAGENET), p)
    got = out.float().cpu().numpy()
    assert np.array_equal(got, _bf16_of(ref) if bf16 else ref)


@pytest.mark.parametrize("fmt", ["rgb", "bgra"])
@pytest.mark.parametrize("shape", [(2, 480, 640, 224, 224, 16), (2, 33, 47, 16, 16, 4)])
def test_packed_patch_layout_equals_oracle_patchified(ctx, fmt, shape):
    B, H, W, oh, ow, p = shape
    C = 4 if fmt.endswith("a") else 3
    rng = np.random.default_rng(zlib.crc32(repr(("packedp", fmt, shape)).encode()))
    frames = rng.integers(0, 256, (B, H, W, C), dtype=np.uint8)
    cfg = L.ImagePreprocess.make(oh, ow, **IMAGENET)
    out = torch.full((B, (oh // p) * (ow // p), 3 * p * p), 7.0, device="cuda")
    torch.cuda.synchronize()
    L.preprocess_packed_patches_device(ctx, torch.from_numpy(frames).cuda(), B, H, W, fmt, cfg, p, out)
    ctx.synchronize()
    ref = _patchify(O.preprocess_packed(frames, L.PACKED_FORMATS[fmt], oh, ow, **IMAGENET), p)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_patch_layout_rejects_sizes_it_does_not_divide(ctx):
    y = torch.zeros((1, 32, 32), dtype=torch.uint8, device="cuda")
    uv = torch.zeros((1, 16, 16, 2), dtype=torch.uint8, device="cuda")
    out = torch.zeros((1, 64, 48), device="cuda")
    with pytest.raises(L.LwmError, match="must divide the output size"):
        L.preprocess_nv12_patches_device(ctx, y, uv, 1, 32, 32, 0, L.ImagePreprocess.make(30, 30), 4, out)
