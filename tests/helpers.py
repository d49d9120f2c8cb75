"""Shared helpers for the parity tests: seeded inputs and host views of device buffers."""
import numpy as np

QK = 32


def align256(n):
    return (n + 255) & ~255


def act_planes_host(buf, n_tok, cols):
    """Split a device Q8_0 activation buffer (copied to host uint8) into its planes."""
    b = np.asarray(buf).view(np.uint8)
    nb = cols // QK
    o = 0
    qs = b[o:o + n_tok * cols].view(np.int8).reshape(n_tok, cols)
    o += align256(n_tok * cols)
    dh = b[o:o + n_tok * nb * 2].view(np.uint16).reshape(n_tok, nb)
    o += align256(n_tok * nb * 2)
    d = b[o:o + n_tok * nb * 4].view(np.float32).reshape(n_tok, nb)
    o += align256(n_tok * nb * 4)
    s = b[o:o + n_tok * nb * 4].view(np.int32).reshape(n_tok, nb)
    return qs, dh, d, s


def blocks_to_planes(blocks, n_tok, cols):
    """ggml block_q8_0 bytes -> (qs int8 [n_tok][cols], d bits uint16 [n_tok][nb])."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(n_tok, cols // QK, 34)
    dh = (b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8))
    qs = b[:, :, 2:].reshape(n_tok, cols).view(np.int8)
    return qs, dh


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def random_weights(rng, rows, cols, sigma=0.02):
    return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)).astype(np.float32)
