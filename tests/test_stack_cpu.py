"""Projection-stack host logic on the CPU (tinygrad_dx12_b200/stack.py): packed row / K-column
shards against slices of the oracle's dequant, the unsharded chain against the oracle chain,
and the tensor-parallel chain on two gloo ranks (column-parallel q/k/v/gate/up, row-parallel
o/down with an fp32 all-reduce) against the unsharded oracle."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch

from oracle import packed_ref as ref
from tests.stack_helpers import CONFIGS, OracleOps, gloo_worker, initial_h, oracle_forward, spec_of, to_numpy
from tinygrad_dx12_b200 import stack as S


def _dq(w):
    s = spec_of(w)
    return ref.dequant(s.data, s.format, s.shape, s.scales, s.block_size, "float32", s.scale_dtype)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_shards_are_dequant_slices(name):
    cfg = CONFIGS[name]
    w = S.make_matrix(cfg, 1, "down", "cpu")  # (hidden, inter)
    full = _dq(w)
    n, k = w.shape
    np.testing.assert_array_equal(_dq(S.shard_rows(w, 64, 192)), full[64:192])
    np.testing.assert_array_equal(_dq(S.shard_cols(w, 128, 384)), full[:, 128:384])
    cat = S.concat_rows([S.shard_rows(w, 0, 32), S.shard_rows(w, 100, 132)])
    np.testing.assert_array_equal(_dq(cat), np.concatenate([full[0:32], full[100:132]]))


def test_misaligned_shards_rejected():
    cfg = CONFIGS["int4"]
    w = S.make_matrix(cfg, 0, "o", "cpu")
    with pytest.raises(ValueError):
        S.shard_cols(w, 16, 48)  # not on a 32-wide scale block
    with pytest.raises(ValueError):
        S.split(100, 3, 0)
    wide = S.StackConfig(hidden=256, q_dim=96, kv_dim=32, inter=512, layers=1, fmt="int4", block=32, scale="f16u",
                         act=torch.float16)
    with pytest.raises(ValueError):  # 96 / 2 = 48 rows of q: o's K shard is not block-aligned
        S.shard_layer({p: S.make_matrix(wide, 0, p, "cpu") for p in wide.proj_shapes()}, wide, 0, 2)


def _close(y, r, act):
    tol = 4e-3 if act == torch.bfloat16 else 1e-3
    rel_f = np.linalg.norm(y - r) / np.linalg.norm(r)
    assert rel_f <= tol, rel_f
    assert np.all(np.isfinite(y))


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_unsharded_chain_matches_oracle(name):
    cfg = CONFIGS[name]
    st = S.TPStack(cfg, 0, 1, device="cpu", ops=OracleOps())
    h = st.forward(initial_h(cfg, 3))
    _close(to_numpy(h), oracle_forward(cfg, initial_h(cfg, 3)), cfg.act)


@pytest.mark.parametrize("name", ["int4", "fp4"])
def test_tensor_parallel_two_gloo_ranks(name, tmp_path):
    import torch.multiprocessing as mp

    cfg = CONFIGS[name]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(gloo_worker, args=(2, port, name, 2, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r = oracle_forward(cfg, initial_h(cfg, 2))
    y0, y1 = np.load(tmp_path / "rank0.npy"), np.load(tmp_path / "rank1.npy")
    np.testing.assert_array_equal(y0, y1)  # h is replicated after every all-reduce
    _close(y0, r, cfg.act)
