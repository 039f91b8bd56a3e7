"""Sign vector of the randomized Hadamard transform (RHT) the int4 and k8v4 caches are stored in.

The stock vLLM `single_rht` (called by the plugin at vllm_quantpack/attention/int4_kv.py:326,329 and
k8v4_kv.py:71-72) keeps its sign vector inside vLLM >= 0.31. This build defines its own: d_i = -1 where bit 63 of
splitmix64(seed * 2**32 + i) is set, seed 0. The transform is y = H (d * x) with H the unnormalised Sylvester
Hadamard matrix; the inverse is d * (H y), and inverse(forward(x)) = head * x, so attention scores take
softmax_scale / head and outputs are divided by head (int4_kv.py:328-329). A cache written with one sign vector must
be read with the same one."""
import functools

import numpy as np

SEED = 0
_M64 = (1 << 64) - 1


def _splitmix64(z):
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


@functools.lru_cache(maxsize=None)
def sign_bits(head_size, seed=SEED):
    """uint32 words, bit i set where d_i = -1 (the layout the kernels take)."""
    if head_size <= 0 or head_size & (head_size - 1):
        raise ValueError(f"RHT head size must be a power of two, got {head_size}")
    words = np.zeros((head_size + 31) // 32, dtype=np.uint32)
    for i in range(head_size):
        if _splitmix64((seed << 32) + i) >> 63:
            words[i // 32] |= np.uint32(1 << (i % 32))
    words.flags.writeable = False
    return words


_device_bits = {}


def device_sign_bits(head_size, device):
    """The sign words as an int32 tensor on `device` (cached; the first call per device copies from the host, so make
    it before any CUDA-graph capture)."""
    import torch
    key = (head_size, str(torch.device(device)))
    t = _device_bits.get(key)
    if t is None:
        t = torch.from_numpy(sign_bits(head_size).view(np.int32).copy()).to(device)
        _device_bits[key] = t
    return t
