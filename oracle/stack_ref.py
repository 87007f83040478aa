"""CPU restatement of the packed projection-stack chain -- TEST INFRASTRUCTURE ONLY.

Only tests, the smoke check and the benchmark's CPU leg may import this module; the product
path (tinygrad_dx12_b200.stack) never does. It runs the chain of
``tinygrad_dx12_b200/stack.py`` unsharded, with every packed projection through
``packed_ref.packed_linear_ref`` (the reference's CPU matmul branch, tinygrad-dx12
``codegen/linalg.py:169-174``: decode to fp32, fp32 matmul) and the same rounding points:

    x = rnd(rmsnorm(h))                       rmsnorm in fp32, eps 1e-6
    q = rnd(x Wq^T)                           (k, v do not reach the output)
    h = rnd(h + x' Wo^T)   with x' = q, fp32 partial
    x = rnd(rmsnorm(h)); g = rnd(x Wg^T); u = rnd(x Wu^T); m = rnd(g * u)
    h = rnd(h + m Wd^T);   x = rnd(rmsnorm(h))

where rnd() rounds to the activation dtype.
"""

from __future__ import annotations

import numpy as np

from . import packed_ref as ref

EPS = 1e-6


def rnd(a: np.ndarray, act: str) -> np.ndarray:
    return ref.cast(np.asarray(a, np.float32), act).astype(np.float32)


def rmsnorm(h: np.ndarray) -> np.ndarray:
    h = h.astype(np.float32)
    return h / np.sqrt(np.mean(h * h, axis=-1, keepdims=True, dtype=np.float32) + np.float32(EPS))


def stack_forward(layers: list[dict], h0: np.ndarray, act: str, linear=None) -> np.ndarray:
    """layers: a sequence (``len`` and indexing) holding per layer a dict projection name ->
    PackedSpec (full matrices); a lazy sequence lets full-size layers be built one at a time.
    ``linear(spec, x)`` computes x @ dequant(W)^T in float32 (default: the numpy restatement).
    Returns h (float32 array holding act-dtype values)."""
    linear = linear or ref.packed_linear_ref
    h = rnd(h0, act)
    x = rnd(rmsnorm(h), act)
    for i in range(len(layers)):
        L = layers[i]
        q = rnd(linear(L["q"], x), act)
        h = rnd(h + linear(L["o"], q), act)
        x = rnd(rmsnorm(h), act)
        g = rnd(linear(L["gate"], x), act)
        u = rnd(linear(L["up"], x), act)
        m = rnd(g * u, act)
        h = rnd(h + linear(L["down"], m), act)
        x = rnd(rmsnorm(h), act)
    return h
