"""Tensor-parallel stack on 2 GPUs (one process per GPU, NCCL): the fused peer-memory
reduction (PeerOps) against the NCCL all-reduce path (CudaOps) and the unsharded oracle
chain. Skipped unless at least two GPUs are visible; ranks never share a GPU."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from tests.stack_helpers import CONFIGS, initial_h, to_numpy
    from tinygrad_dx12_b200 import stack as S
    from tinygrad_dx12_b200.packed import PackedTensor

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = CONFIGS["fp4"]

        def mk(layer, proj):
            w = S.make_matrix(cfg, layer, proj, "cpu")
            return PackedTensor(w.data.to(dev), w.format, w.shape, w.scales.to(dev), w.block_size)

        peer = S.PeerOps(rows_max=8, hidden=cfg.hidden)
        outs = {}
        for name, ops in (("nccl", S.CudaOps()), ("peer", peer)):
            st = S.TPStack(cfg, rank, world, device=dev, ops=ops, matrix_fn=mk)
            for rep in range(3):  # several forwards: epochs and both buffers cycle
                h = st.forward(initial_h(cfg, 3).to(dev))
            torch.cuda.synchronize()
            outs[name] = to_numpy(h)
        peer.close()
        np.save(os.path.join(out_dir, f"nccl{rank}.npy"), outs["nccl"])
        np.save(os.path.join(out_dir, f"peer{rank}.npy"), outs["peer"])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_reduce_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    from tests.stack_helpers import CONFIGS, initial_h, oracle_forward

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    cfg = CONFIGS["fp4"]
    r = oracle_forward(cfg, initial_h(cfg, 3))
    p0, p1 = np.load(tmp_path / "peer0.npy"), np.load(tmp_path / "peer1.npy")
    n0 = np.load(tmp_path / "nccl0.npy")
    np.testing.assert_array_equal(p0, p1)  # fixed-order sums: h bitwise replicated
    for y in (p0, n0):
        assert np.all(np.isfinite(y))
        assert np.linalg.norm(y - r) / np.linalg.norm(r) <= 4e-3
