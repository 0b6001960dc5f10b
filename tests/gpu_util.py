"""Shared helpers for the GPU tests (device buffers through torch, which is
used only as a device-memory allocator and stream provider here)."""
import numpy as np

import oracle as O


def rel_l2(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


# Device buffers made by dev() stay referenced until the test ends: a temporary
# whose data_ptr() is passed to a kernel must not return to torch's caching
# allocator before the kernel has been enqueued (a later dev() would reuse it).
ALIVE = []


def dev(a):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    ALIVE.append(t)
    return t


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def make_weights(t, n, k, seed, std=0.02):
    """Quantized weights [n, row_bytes(t, k)] from seeded N(0, std) floats (oracle quantizer)."""
    x = O.randn(seed, n * k, std).reshape(n, k)
    if t == O.Q6_K:  # no quantizer for Q6_K: random bytes with finite, small f16 scales
        rng = np.random.default_rng(seed)
        w = rng.integers(0, 256, size=(n, k // 256, 210), dtype=np.uint8)
        w[..., 208:210] = (rng.standard_normal((n, k // 256)) * 0.001).astype(np.float16).view(np.uint8).reshape(
            n, k // 256, 2)
        return w.reshape(n, -1)
    return O.quantize(t, x)
