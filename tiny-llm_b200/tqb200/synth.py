"""Seeded synthetic tensors and models in the reference's byte layouts.

The reference measures on random seeded tensors (benchmarks/bench_kernels.cpp:54-66)
and random-weight models (tools/make_fake_model.py); there is no dataset on this
path.  Everything here is drawn from numpy's PCG64 ``default_rng(seed)`` and
packed into the exact in-band formats:

* i4: per row, ceil(K/G) groups of ``[scale f16][zero f16][G/2 bytes]``, low
  nibble = even column (runtime/tiny_format.h:66-77).
* VQ2: ``[codebook 256x4 f16][one uint8 index per 4 weights, row-major]``
  (runtime/tiny_format.h:91-103).

``quantize_i4_rtn`` restates the reference exporter's vectorised RTN quantiser
(tools/export_qwen_to_tiny_i4.py:298-352): fp32 min/max per group, scale =
(max-min)/15 and zero = -min/scale rounded to fp16, codes = round(w/s + z)
clipped to [0, 15] using the fp16-rounded s and z.
"""
from __future__ import annotations

import numpy as np

I4_HEADER = 4


def i4_row_bytes(cols: int, group_size: int) -> int:
    return ((cols + group_size - 1) // group_size) * (I4_HEADER + group_size // 2)


def vq2_bytes(rows: int, cols: int) -> int:
    return 2048 + rows * (cols // 4)


def pack_i4(codes: np.ndarray, scale: np.ndarray, zero: np.ndarray, group_size: int) -> np.ndarray:
    """Pack codes [M, K] (0..15), scale/zero [M, ceil(K/G)] into the interleaved layout.

    A partial last group keeps its full G/2-byte slot with the unused nibbles zero,
    as the reference packers do (benchmarks/bench_kernels.cpp:127-165).
    """
    M, K = codes.shape
    G = group_size
    ng = (K + G - 1) // G
    kp = ng * G
    c = np.zeros((M, kp), dtype=np.uint8)
    c[:, :K] = codes.astype(np.uint8) & 0x0F
    c = c.reshape(M, ng, G // 2, 2)
    nib = (c[..., 0] | (c[..., 1] << 4)).astype(np.uint8)          # [M, ng, G/2]
    hdr = np.empty((M, ng, 2), dtype=np.float16)
    hdr[..., 0] = scale.astype(np.float16)
    hdr[..., 1] = zero.astype(np.float16)
    out = np.concatenate([hdr.view(np.uint8).reshape(M, ng, 4), nib], axis=2)
    return np.ascontiguousarray(out.reshape(M, ng * (I4_HEADER + G // 2)))


def unpack_i4(w: np.ndarray, rows: int, cols: int, group_size: int):
    """Inverse of pack_i4: returns (codes [M,K] uint8, scale f16 [M,ng], zero f16 [M,ng])."""
    G = group_size
    ng = (cols + G - 1) // G
    b = np.asarray(w, dtype=np.uint8).reshape(rows, ng, I4_HEADER + G // 2)
    hdr = np.ascontiguousarray(b[:, :, :4]).view(np.float16).reshape(rows, ng, 2)
    nib = b[:, :, 4:]
    codes = np.empty((rows, ng, G), dtype=np.uint8)
    codes[:, :, 0::2] = nib & 0x0F
    codes[:, :, 1::2] = nib >> 4
    return codes.reshape(rows, ng * G)[:, :cols], hdr[..., 0].copy(), hdr[..., 1].copy()


def quantize_i4_rtn(w: np.ndarray, group_size: int, symmetric: bool = False) -> np.ndarray:
    """RTN i4 quantisation of fp32 w [M, K] (K % G == 0), packed."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = w.shape
    G = group_size
    assert K % G == 0, "quantize_i4_rtn needs K % group_size == 0"
    g = w.reshape(M * (K // G), G)
    vmin = g.min(axis=1)
    vmax = g.max(axis=1)
    if symmetric:
        amax = np.maximum(np.abs(vmin), np.abs(vmax))
        scale = np.where(amax == 0.0, np.float32(0.0), amax / np.float32(7.0)).astype(np.float16)
        zero = np.full(scale.shape, 8.0, dtype=np.float16)
        s = scale.astype(np.float32)
        valid = s != 0
        q = np.zeros(g.shape, dtype=np.uint8)
        q[valid] = np.clip(np.round(g[valid] / s[valid, None] + np.float32(8.0)), 0, 15).astype(np.uint8)
    else:
        same = vmax == vmin
        scale_f = np.where(same, np.float32(0.0), (vmax - vmin) / np.float32(15.0)).astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            zero_f = np.where(same, np.float32(0.0), -vmin / scale_f).astype(np.float32)
        scale = scale_f.astype(np.float16)
        zero = zero_f.astype(np.float16)
        s = scale.astype(np.float32)
        z = zero.astype(np.float32)
        valid = (~same) & (s != 0)
        q = np.zeros(g.shape, dtype=np.uint8)
        sv = np.where(valid, s, np.float32(1.0))
        qv = np.round(g / sv[:, None] + z[:, None]).astype(np.int32)
        q[valid] = np.clip(qv[valid], 0, 15).astype(np.uint8)
    ng = K // G
    return pack_i4(q.reshape(M, K), scale.reshape(M, ng), zero.reshape(M, ng), G)


def random_i4(rng: np.random.Generator, rows: int, cols: int, group_size: int,
              scale_sigma: float = 0.02) -> np.ndarray:
    """Config-1 style i4 matrix: codes U{0..15}, scale |N(0,sigma)|/7.5, zero U[0,15] (fp16)."""
    ng = (cols + group_size - 1) // group_size
    codes = rng.integers(0, 16, (rows, cols), dtype=np.uint8)
    scale = (np.abs(rng.normal(0.0, scale_sigma, (rows, ng))) / 7.5).astype(np.float16)
    zero = rng.uniform(0.0, 15.0, (rows, ng)).astype(np.float16)
    return pack_i4(codes, scale, zero, group_size)


def random_i4_fast(rng: np.random.Generator, rows: int, cols: int, group_size: int,
                   scale_sigma: float = 0.02) -> np.ndarray:
    """Same distribution as random_i4 for K % G == 0, drawn byte-wise (two uniform
    nibbles per uniform byte) so multi-GB timing models build in seconds."""
    G = group_size
    assert cols % G == 0
    ng = cols // G
    nib = np.frombuffer(rng.bytes(rows * ng * (G // 2)), dtype=np.uint8).reshape(rows, ng, G // 2)
    hdr = np.empty((rows, ng, 2), dtype=np.float16)
    hdr[..., 0] = (np.abs(rng.normal(0.0, scale_sigma, (rows, ng))) / 7.5).astype(np.float16)
    hdr[..., 1] = rng.uniform(0.0, 15.0, (rows, ng)).astype(np.float16)
    out = np.concatenate([hdr.view(np.uint8).reshape(rows, ng, 4), nib], axis=2)
    return np.ascontiguousarray(out.reshape(rows, ng * (4 + G // 2)))


def config1_matvec(seed: int = 0, rows: int = 4864, cols: int = 896, group_size: int = 64):
    """W [4864 x 896] g64 i4, x [896] ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    ng = (cols + group_size - 1) // group_size
    codes = rng.integers(0, 16, (rows, cols), dtype=np.uint8)
    scale = (np.abs(rng.normal(0.0, 0.02, (rows, ng))) / 7.5).astype(np.float16)
    zero = rng.uniform(0.0, 15.0, (rows, ng)).astype(np.float16)
    x = rng.normal(0.0, 1.0, cols).astype(np.float32)
    return pack_i4(codes, scale, zero, group_size), x


def random_vq2(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """Codebook 256x4 fp16 ~ N(0,1) followed by uniform uint8 indices."""
    cb = rng.normal(0.0, 1.0, (256, 4)).astype(np.float16)
    idx = rng.integers(0, 256, (rows, cols // 4), dtype=np.uint8)
    return np.concatenate([cb.view(np.uint8).reshape(-1), idx.reshape(-1)])


def config3_vq2(seed: int = 0, rows: int = 3072, cols: int = 1024):
    """BASELINE config 3 (reference semantics): VQ2 W, x ~ N(0,1), BiIP sign/scale."""
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, 256, (rows, cols // 4), dtype=np.uint8)
    cb = rng.normal(0.0, 1.0, (256, 4)).astype(np.float16)
    x = rng.normal(0.0, 1.0, cols).astype(np.float32)
    sign = rng.choice(np.array([-1.0, 1.0], dtype=np.float32), cols)
    scale = (np.abs(rng.normal(0.0, 1.0, cols)) + 1e-3).astype(np.float32)
    w = np.concatenate([cb.view(np.uint8).reshape(-1), idx.reshape(-1)])
    return w, x, sign, scale


def hadamard_block_size(dim: int) -> int:
    """find_hadamard_block_size (runtime/qwen_model.cpp:61-67)."""
    for bs in (256, 128, 64, 32, 16, 8, 4, 2):
        if dim % bs == 0:
            return bs
    return 1


GPTQ_MAGIC = 0x47505451  # 'GPTQ' little-endian (runtime/tiny_format.h:135)


def random_gptq(rng: np.random.Generator, rows: int, cols: int, group_size: int,
                act_order: bool = False) -> np.ndarray:
    """A GPTQ-INT4 tensor in the reference's in-band layout (runtime/tiny_format.h:108-182):
    [magic][flags][scales f16 [ng][rows]][qzeros f16 [ng][rows]][g_idx u32 [cols] when
    act_order][qweight u32 [cols/8][rows], column k of a word in bits 4k..4k+3].  Codes
    U{0..15}, scales |N(0,0.02)|/7.5, zeros U[0,15] (stored as the real zero point);
    act-order assigns the columns to groups by a seeded permutation."""
    G = group_size
    assert cols % G == 0 and cols % 8 == 0
    ng = cols // G
    hdr = np.array([GPTQ_MAGIC, 1 if act_order else 0], np.uint32).view(np.uint8)
    scales = (np.abs(rng.normal(0.0, 0.02, (ng, rows))) / 7.5).astype(np.float16).view(np.uint8)
    zeros = rng.uniform(0.0, 15.0, (ng, rows)).astype(np.float16).view(np.uint8)
    parts = [hdr, scales.ravel(), zeros.ravel()]
    if act_order:
        g_idx = (rng.permutation(cols) // G).astype(np.uint32)
        parts.append(g_idx.view(np.uint8))
    qw = np.frombuffer(rng.bytes(cols // 8 * rows * 4), np.uint32)
    parts.append(qw.view(np.uint8))
    return np.ascontiguousarray(np.concatenate(parts))
