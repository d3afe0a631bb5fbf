"""CPU-only checks of the native boundary: the C-ABI library loads and exports
every symbol include/klab_b200.h declares, host-side logic (codec, validation,
planning constants) behaves, and the registered ops keep their contracts under
FakeTensorMode. No GPU work is launched here."""

import ctypes as ct
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import codec as oc

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "klab_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"KLAB_API\s+[\w\s\*]*?\b((?:klab|lab)_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from klab_b200 import _native

    lib = _native.lib()
    declared = declared_symbols()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(lib, name), name
        assert name in _native.EXPORTED, f"{name} declared but not bound in _native"
    raw = ct.CDLL(str(_native.LIB_PATH))
    for name in declared:
        getattr(raw, name)
    assert _native.lib().klab_version() == 1


def test_alias_and_cubin_present():
    from klab_b200 import _native

    assert (_native.LIB_DIR / "libkernel_lab.so").resolve() == _native.LIB_PATH.resolve()
    assert _native.PREFETCH_CUBIN.stat().st_size > 0


def test_error_strings_and_options():
    from klab_b200 import _native

    assert "Invalid" in _native.error_string(_native.E_INVALID)
    assert "Shape" in _native.error_string(_native.E_SHAPE)
    assert _native.lib().lab_error_string(-1000).decode().startswith("Cannot load CUDA driver")
    for opt, values in ((_native.OPT_SPLIT, (-1, 0, 1)), (_native.OPT_PDL, (0, 1)), (_native.OPT_GENERIC, (1, 0)),
                        (_native.OPT_TENSOR, (0, 2, 3, 1)), (_native.OPT_CTAS_PER_SM, (1, 0)),
                        (_native.OPT_PROLOGUE, (0x00, 0x02, 0x10, 0x31, -1)), (_native.OPT_MAX_TILE, (8, 1, 2, 4))):
        before = _native.get_option(opt)
        for v in values:
            _native.set_option(opt, v)
            assert _native.get_option(opt) == v
        _native.set_option(opt, before)
    assert _native.lib().klab_set_option(_native.OPT_SPLIT, 7) == _native.E_INVALID
    for bad in (0x04, 0x40, 0x100, -2):  # each part of the prologue option is 0..3
        assert _native.lib().klab_set_option(_native.OPT_PROLOGUE, bad) == _native.E_INVALID
    assert _native.get_option(_native.OPT_PROLOGUE) == -1
    for bad in (0, 3, 16):
        assert _native.lib().klab_set_option(_native.OPT_MAX_TILE, bad) == _native.E_INVALID
    assert _native.get_option(_native.OPT_MAX_TILE) == 4


def test_invalid_arguments_rejected_before_any_device_work():
    from klab_b200 import _native

    lib = _native.lib()
    assert lib.klab_gemv(0, 0, None, 64, None, None, None, None, 8, 0, 1, 8, 64, None, 0, None) == _native.E_INVALID
    assert lib.klab_raw_linear(None, None, None, 0, 1, 1, 1, None, 0, None) == _native.E_INVALID
    assert lib.lab_launch(None, 1, 1, 32, None, None) == _native.E_INVALID
    assert lib.lab_load_ptx(None, None) == _native.E_INVALID
    assert lib.klab_int8_linear(None, 0, None, None, 32, None, 0, 1, 1, 64, None, 0, None) == _native.E_UNSUPPORTED
    assert lib.klab_residual_rmsnorm(None, None, None, None, 1, 64, 1e-6, None) == _native.E_INVALID
    assert lib.klab_add_rmsnorm(None, None, None, None, None, 1, 64, 1e-6, None) == _native.E_INVALID
    assert lib.klab_silu_mul(None, None, 1, 64, None) == _native.E_INVALID
    assert lib.klab_add_rmsnorm_linear(None, None, None, 1e-6, None, None, None, 1, 8, 64, None, 0, None) \
        == _native.E_INVALID
    assert lib.klab_silu_mul_linear(None, None, None, 1, 8, 64, None, 0, None) == _native.E_INVALID
    assert lib.klab_decode_attention(None, None, None, None, None, None, None, 0, None, None, 0, 64, 8, 2, 0.125,
                                     None) == _native.E_INVALID
    fake = 16  # never dereferenced: the shape checks reject these calls first
    assert lib.klab_residual_rmsnorm(fake, fake, fake, fake, 1, 8193, 1e-6, None) == _native.E_SHAPE
    assert lib.klab_residual_rmsnorm(fake, fake, fake, fake, 1, 64, 0.0, None) == _native.E_INVALID
    assert lib.klab_add_rmsnorm(fake, fake, fake, fake, fake, 1, 63, 1e-6, None) == _native.E_SHAPE
    assert lib.klab_silu_mul(fake, fake, 1, 63, None) == _native.E_SHAPE
    assert lib.klab_add_rmsnorm_linear(fake, fake, fake, 1e-6, fake, fake, None, 1, 8, 60, None, 0, None) \
        == _native.E_SHAPE
    assert lib.klab_silu_mul_linear(fake, fake, fake, 1, 8, 60, None, 0, None) == _native.E_SHAPE
    # Fused add+RMSNorm: an in-place residual update (x_out over res or y) or an out over the
    # inputs is rejected before launch; the addresses are never dereferenced.
    res, y, nw, w, out, xo = 1 << 20, 2 << 20, 3 << 20, 4 << 20, 5 << 20, 6 << 20
    for bad in ((res, y, nw, w, out, res), (res, y, nw, w, out, y + 64), (res, y, nw, w, res, xo),
                (res, y, nw, w, out, out)):
        assert lib.klab_add_rmsnorm_linear(bad[0], bad[1], bad[2], 1e-6, bad[3], bad[4], bad[5], 2, 8, 64, None, 0,
                                           None) == _native.E_INVALID, bad
    assert lib.klab_silu_mul_linear(res, w, res + 128, 2, 8, 64, None, 0, None) == _native.E_INVALID
    assert lib.klab_decode_attention(fake, fake, fake, fake, fake, fake, fake, 1 << 20, fake, None, 0, 64, 34, 2,
                                     0.125, None) == _native.E_SHAPE  # 17 query heads per kv head
    assert lib.klab_decode_attention(fake, fake, fake, fake, fake, fake, fake, 1 << 20, fake, None, 64, 64, 8, 2,
                                     0.125, None) == _native.E_SHAPE  # len + 1 > capacity
    assert lib.klab_decode_attention(fake, fake, fake, fake, fake, fake, fake, 1 << 20, fake, fake, 0, 65537, 8, 2,
                                     0.125, None) == _native.E_SHAPE  # capacity above 65536


def test_workspace_sizes():
    from klab_b200 import _native

    lib = _native.lib()
    assert lib.klab_gemv_workspace_bytes(_native.W_BF16, 1, 4096, 2048) == 0  # a single chunk never splits
    need = lib.klab_gemv_workspace_bytes(_native.W_BF16, 1, 512, 14336)
    assert need >= 512 * 7 * 4 + 512 * 4


@pytest.mark.parametrize("m", [1, 2, 4, 8, 9, 16])
def test_workspace_covers_the_token_tiles(m):
    """INT8 per-row and E2M1 weights at M <= 16 may run as warp-level tensor-core token tiles,
    which keep FP32 phase partials [row group][phase][M][16] after the 64 KiB of tickets
    (phases of 1024 INT8 / 2048 E2M1 columns): the advertised workspace holds them."""
    from klab_b200 import _native

    lib = _native.lib()
    for wfmt, ks in ((_native.W_I8_ROW, 1024), (_native.W_FP4_G32H, 2048)):
        for n, k in ((14336, 4096), (8192, 8192), (100, 2048), (4100, 2560)):
            groups, phases = -(-n // 16), -(-k // ks)
            assert lib.klab_gemv_workspace_bytes(wfmt, m, n, k) >= 65536 + groups * phases * m * 16 * 4, (wfmt, n, k)


@pytest.mark.parametrize("shape", [(1024, 64), (3, 129), (48, 320), (5, 1), (2, 4096)])
def test_host_codec_matches_oracle(shape):
    from klab_b200 import compressed_bf16 as cb

    rng = np.random.default_rng(sum(shape))
    bits = rng.integers(0, 65536, size=shape, dtype=np.uint64).astype(np.uint16)
    if shape[0] > 2:
        bits[1] = 0x3F80 + (rng.integers(0, 64, size=shape[1]).astype(np.uint16))  # coded rows
    mine, ref = cb.pack_bits(bits), oc.pack_bits(bits)
    np.testing.assert_array_equal(mine.metadata, ref.metadata)
    np.testing.assert_array_equal(mine.payload, ref.payload)
    assert mine.source_sha256 == ref.source_sha256
    np.testing.assert_array_equal(cb.unpack_bits(mine), bits)
    cb.validate(mine)


def test_host_codec_rejects_corruption():
    from klab_b200 import compressed_bf16 as cb

    packed = cb.pack_bits(np.full((1, 64), 0x3F80, dtype=np.uint16))
    bad = cb.PackedCPU(packed.payload, packed.metadata | np.uint32(1), 1, 64, packed.source_sha256)
    with pytest.raises(ValueError):
        cb.unpack_bits(bad)
    bad = cb.PackedCPU(packed.payload[:95], packed.metadata, 1, 64, packed.source_sha256)
    with pytest.raises(ValueError):
        cb.unpack_bits(bad)
    overflow = np.zeros(96, np.uint8)
    overflow[1] = 1
    bad = cb.PackedCPU(overflow, np.array([255 << 23], dtype="<u4"), 1, 64, packed.source_sha256)
    with pytest.raises(ValueError):
        cb.unpack_bits(bad)
    wrong_digest = cb.PackedCPU(packed.payload, packed.metadata, 1, 64, "0" * 64)
    with pytest.raises(ValueError):
        cb.validate(wrong_digest)
    for value in (np.ones((1, 64), dtype=np.float32), np.empty((0, 64), dtype=np.uint16), np.ones(64, np.uint16)):
        with pytest.raises(ValueError):
            cb.pack_bits(value)


def test_mtile_table_matches_reference_fixture():
    from klab_b200 import mtile_bf16 as mt

    golden = np.load(ROOT / "tests" / "golden" / "reference_codec.npz")
    for m, tile in zip(golden["tile__m"], golden["tile__tile"]):
        assert mt.tile_for_m(int(m)) == int(tile)
    assert len(mt.kernel_names()) == int(golden["tile__kernel_count"]) == 128
    for bad in (0, -1, 65536, True, 1.5):
        with pytest.raises(ValueError):
            mt.tile_for_m(bad)


def test_fake_tensor_contracts():
    from torch._subclasses.fake_tensor import FakeTensorMode

    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import fp4, half_projection, int8_weights, kernel_lab  # noqa: F401  (registers ops)

    with FakeTensorMode():
        x = torch.empty(3, 128, dtype=torch.bfloat16)
        payload = torch.empty(2 * 4 * 96, dtype=torch.uint8)
        metadata = torch.empty(4 * 2, dtype=torch.int32)
        y = torch.ops.compressed_bf16.compressed_linear(x, payload, metadata, 4, 128, 128, 8, "bf16")
        assert tuple(y.shape) == (3, 4) and y.dtype == torch.bfloat16
        with pytest.raises(ValueError):
            torch.ops.compressed_bf16.compressed_linear(x, payload, metadata, 5, 128, 128, 8, "bf16")
        y = torch.ops.kernel_lab.int8_linear(torch.empty(2, 64, dtype=torch.float16),
                                             torch.empty(7, 64, dtype=torch.int8), torch.empty(7, 1))
        assert tuple(y.shape) == (2, 7) and y.dtype == torch.float32
        y = torch.ops.kernel_lab.half_linear(torch.empty(2, 64, dtype=torch.bfloat16),
                                             torch.empty(5, 64, dtype=torch.bfloat16))
        assert tuple(y.shape) == (2, 5) and y.dtype == torch.float32
        y = torch.ops.kernel_lab.residual_rmsnorm(torch.empty(3, 96), torch.empty(3, 96), torch.empty(96), 1e-5)
        assert tuple(y.shape) == (3, 96) and y.dtype == torch.float32
    assert cb.kernel_names()[-1] == "cbf16_unpack" and len(cb.kernel_names()) == 33
