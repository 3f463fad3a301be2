"""Seeded inputs for the projection (k-quant matvec) tests, generated the way
the reference's own kernel tests generate theirs
(crates/llm-core/tests/kernels.rs:44-101): the same xorshift64* stream, the
same block construction (random bytes, f16 scales of bounded magnitude), the
same activation draw and the same shape lists; and that file's f64 reference
(kernels.rs:119-190): dequantize the weight row and the int8 activations and
sum in f64, with the sum of |terms| as the scale of the allowed drift."""
from __future__ import annotations

import numpy as np

import oracle as orc

Q8_0, Q4_K, Q6_K = orc.Q8_0, orc.Q4_K, orc.Q6_K
TYPES = (Q4_K, Q6_K, Q8_0)
BLOCK_LEN = {Q4_K: 256, Q6_K: 256, Q8_0: 32}
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34}

# (k, rows), kernels.rs:23-35 and :37-44
AWKWARD_SHAPES = [(256, 1), (1, 1), (32, 3), (37, 3), (255, 2), (257, 2), (300, 4), (512, 5),
                  (8192, 2), (16384, 1)]
MODEL_SHAPES = [(2560, 8192), (2560, 9216), (9216, 2560), (4096, 2560), (2560, 1024)]

_M64 = (1 << 64) - 1


class XorShift:
    """The reference tests' xorshift64* (kernels.rs:48-72); the raw stream
    comes from the oracle's C loop, the byte and signed mappings are these."""

    def __init__(self, seed: int):
        self.state = np.array([(seed | 1) & _M64], np.uint64)

    def raw(self, n: int) -> np.ndarray:
        return orc.xorshift_stream(self.state, n)

    @staticmethod
    def as_bytes(raw: np.ndarray) -> np.ndarray:
        return ((raw >> np.uint64(33)) & np.uint64(0xFF)).astype(np.uint8)

    @staticmethod
    def as_signed(raw: np.ndarray) -> np.ndarray:
        # (next >> 40) as f32 / 2^23 - 1.0, in f32
        v = (raw >> np.uint64(40)).astype(np.float32) / np.float32(1 << 23)
        return (v - np.float32(1.0)).astype(np.float32)

    def signed(self) -> np.float32:
        return self.as_signed(self.raw(1))[0]

    def signed_n(self, n: int) -> np.ndarray:
        return self.as_signed(self.raw(n))


def _f16_bytes(x: np.ndarray) -> np.ndarray:
    """[n] f32 -> [n][2] little-endian f16 bytes (round to nearest even)."""
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def random_weights(ty: int, rng: XorShift, n: int) -> np.ndarray:
    """n blocks of well-formed weights (kernels.rs:75-101), in its draw order:
    Q4_K d, dmin, 140 bytes; Q6_K 208 bytes, d; Q8_0 d, 32 bytes."""
    if ty == Q4_K:
        raw = rng.raw(n * 142).reshape(n, 142)
        d = _f16_bytes(XorShift.as_signed(raw[:, 0]) * np.float32(0.05))
        dmin = _f16_bytes(XorShift.as_signed(raw[:, 1]) * np.float32(0.02))
        a = np.concatenate([d, dmin, XorShift.as_bytes(raw[:, 2:])], axis=1)
    elif ty == Q6_K:
        raw = rng.raw(n * 209).reshape(n, 209)
        d = _f16_bytes(XorShift.as_signed(raw[:, 208]) * np.float32(0.01))
        a = np.concatenate([XorShift.as_bytes(raw[:, :208]), d], axis=1)
    else:
        raw = rng.raw(n * 33).reshape(n, 33)
        d = _f16_bytes(XorShift.as_signed(raw[:, 0]) * np.float32(0.05))
        a = np.concatenate([d, XorShift.as_bytes(raw[:, 1:])], axis=1)
    a = np.ascontiguousarray(a, np.uint8).reshape(-1)
    assert a.size == n * BLOCK_BYTES[ty]
    return a


def shape_case(ty: int, k: int, rows: int, seed: int):
    """check_shape's inputs (kernels.rs:199-205): the weights, then x."""
    nb = -(-k // BLOCK_LEN[ty])
    rng = XorShift(seed)
    w = random_weights(ty, rng, nb * rows)
    x = (rng.signed_n(k) * np.float32(3.0)).astype(np.float32)
    return w, x


def _f16(b, off):
    return np.frombuffer(bytes(b[off:off + 2]), np.float16)[0].astype(np.float32)


def _scale_min(j, s):
    if j < 4:
        return s[j] & 63, s[j + 4] & 63
    return (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4), (s[j + 4] >> 4) | ((s[j] >> 6) << 4)


def dequantize(ty: int, row: np.ndarray, nblocks: int) -> np.ndarray:
    """kernels.rs:119-165, in f32 as there."""
    out = []
    bb = BLOCK_BYTES[ty]
    for ib in range(nblocks):
        b = row[ib * bb:(ib + 1) * bb]
        if ty == Q4_K:
            d, dmin = _f16(b, 0), _f16(b, 2)
            scales, qs = b[4:16], b[16:]
            for j in range(8):
                sc, m = _scale_min(j, scales)
                ds, ms = np.float32(d * np.float32(sc)), np.float32(dmin * np.float32(m))
                byte = qs[(j // 2) * 32:(j // 2) * 32 + 32]
                q = (byte & 0xF) if j % 2 == 0 else (byte >> 4)
                out.append((ds * q.astype(np.float32) - ms).astype(np.float32))
        elif ty == Q6_K:
            d = _f16(b, 208)
            for n in range(2):
                ql, qh, sc = b[n * 64:], b[128 + n * 32:], b[192 + n * 8:]
                half = np.zeros(128, np.float32)
                for l in range(32):
                    is_ = l // 16
                    q1 = int((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32
                    q2 = int((ql[32 + l] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32
                    q3 = int((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32
                    q4 = int((ql[32 + l] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32
                    s = sc[:8].astype(np.int8).astype(np.float32)
                    half[l] = d * s[is_] * np.float32(q1)
                    half[32 + l] = d * s[is_ + 2] * np.float32(q2)
                    half[64 + l] = d * s[is_ + 4] * np.float32(q3)
                    half[96 + l] = d * s[is_ + 6] * np.float32(q4)
                out.append(half)
        else:
            d = _f16(b, 0)
            out.append((d * b[2:].astype(np.int8).astype(np.float32)).astype(np.float32))
    return np.concatenate(out)


def reference_dot(ty: int, row: np.ndarray, d, qs, k: int):
    """kernels.rs:177-190: (f64 dot, f64 sum of |terms|) of the dequantized
    row and activations (qs * d per super-block, the first k)."""
    w = dequantize(ty, row, -(-k // BLOCK_LEN[ty])).astype(np.float64)
    x = (qs.astype(np.float32) * d[:, None]).astype(np.float32).reshape(-1)[:k].astype(np.float64)
    terms = w[:k] * x
    return float(terms.sum()), float(np.abs(terms).sum())
