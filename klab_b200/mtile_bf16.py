"""M-tiled exact BF16 projections (drop-in for the reference's mtile_bf16.py).

tile_for_m keeps the reference's deterministic rule (mtile_bf16.py:42-52); the
B200 kernel tiles tokens the same way (1, 2, 4, 8 per tile; larger M runs
several tiles), and every token of a tile is bit-identical to the same token
computed alone, as the reference guarantees for R2 vs R1
(verification/verify_mtile_bf16.py:26-45).
"""

from __future__ import annotations

import numbers

REVISION = 2
THREADS = (32, 64, 128, 256)
VECTORS = (2, 8)
OUTPUTS = ("bf16", "fp32")
TILES = (2, 4, 8, 16)
MAX_M = 65535
TILE_RULE = "M == 1 delegates to compressed_bf16; else min(16, smallest power of two >= M)"


def tile_for_m(m):
    """Deterministic token tile: 1 for M == 1, else min(16, next power of two >= M)."""
    if isinstance(m, bool) or not isinstance(m, numbers.Integral):
        raise ValueError("m must be an integer")
    m = int(m)
    if not 1 <= m <= MAX_M:
        raise ValueError(f"m must be in [1, {MAX_M}]")
    tile = 1
    while tile < m and tile < TILES[-1]:
        tile *= 2
    return tile


def kernel_names():
    """The reference's M-tile kernel name set (mtile_kernels.cu:122-144)."""
    return tuple(f"mtbf16_{kind}_{output}_t{threads}_v{vector}_m{tile}"
                 for kind in ("raw", "coded") for output in OUTPUTS
                 for vector in VECTORS for threads in THREADS for tile in TILES)


def get_module(device=None):
    from . import compressed_bf16 as cb

    return cb.get_module(device)


def implementation_fingerprint(device=None):
    from . import compressed_bf16 as cb

    return {"revision": REVISION, "tile_rule": TILE_RULE, "kernel_names": list(kernel_names()),
            "compressed_bf16": cb.implementation_fingerprint(device)}


def _single_token(x):
    import torch

    return isinstance(x, torch.Tensor) and x.ndim == 2 and x.shape[0] == 1


def fused_linear(x, packed, *, threads, vector, output_dtype, out=None):
    """out[M,N] = x[M,K] @ W.T over a compressed_bf16.PackedBF16, tiled over M."""
    from . import compressed_bf16 as cb

    if not isinstance(packed, cb.PackedBF16):
        raise ValueError("packed must come from compressed_bf16.upload()")
    if _single_token(x):
        return cb.fused_linear(x, packed, threads=threads, vector=vector, output_dtype=output_dtype, out=out)
    tile_for_m(x.shape[0] if hasattr(x, "shape") and len(x.shape) == 2 else 0)
    return cb.fused_linear(x, packed, threads=threads, vector=vector, output_dtype=output_dtype, out=out)


def raw_linear(x, w, *, threads, vector, output_dtype, out=None):
    """Same tiling as fused_linear over an uncompressed BF16 w[N,K]."""
    from . import compressed_bf16 as cb

    if not _single_token(x) and hasattr(x, "shape") and len(x.shape) == 2:
        tile_for_m(x.shape[0])
    return cb.raw_linear(x, w, threads=threads, vector=vector, output_dtype=output_dtype, out=out)
