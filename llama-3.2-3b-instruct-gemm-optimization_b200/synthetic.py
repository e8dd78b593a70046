"""Seeded synthetic inputs for the Llama-3.2-3B decode MLP shapes.

No checkpoint or dataset is involved: every tensor is drawn from
``numpy.random.default_rng(seed)``.

* weights ~ N(0, 0.02): ``standard_normal(shape, float32) * 0.02`` -> fp16,
  stored [K, N] (the reference's row-major layout, kernels/gemv_fp8.cu:93).
* activations ~ N(0, 1) fp16.
* FP16 GEMV benchmark case: one generator with seed 0 draws W [3072, 8192]
  first, then x [1, 3072].
* stack layer l: gate, up, down weights from seeds 1000+3l, 1000+3l+1,
  1000+3l+2; the input hidden state from seed 7.
"""
from __future__ import annotations

import numpy as np

HIDDEN = 3072
INTERMEDIATE = 8192
N_LAYERS = 28
RMS_EPS = 1e-5
W_STD = 0.02


def weights(seed: int, K: int, N: int, rng=None) -> np.ndarray:
    rng = np.random.default_rng(seed) if rng is None else rng
    return (rng.standard_normal((K, N), dtype=np.float32) * np.float32(W_STD)).astype(np.float16)


def activations(seed: int, M: int, K: int, rng=None) -> np.ndarray:
    rng = np.random.default_rng(seed) if rng is None else rng
    return rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)


def cfg0_fp16_gemv(K: int = HIDDEN, N: int = INTERMEDIATE):
    """FP16 GEMV y = x W, M=1, seed 0: returns (W [K,N] fp16, x [1,K] fp16)."""
    rng = np.random.default_rng(0)
    W = weights(0, K, N, rng)
    x = activations(0, 1, K, rng)
    return W, x


def layer_seeds(layer: int):
    base = 1000 + 3 * layer
    return base, base + 1, base + 2


def layer_weights(layer: int, hidden: int = HIDDEN, inter: int = INTERMEDIATE):
    """(Wg [hidden, inter], Wu [hidden, inter], Wd [inter, hidden]) fp16."""
    sg, su, sd = layer_seeds(layer)
    return weights(sg, hidden, inter), weights(su, hidden, inter), weights(sd, inter, hidden)


def hidden_state(M: int, hidden: int = HIDDEN, seed: int = 7) -> np.ndarray:
    return activations(seed, M, hidden)
