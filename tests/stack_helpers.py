"""Stack test support: oracle-backed compute for TPStack on CPU tensors, conversions from
PackedTensor to oracle specs, and the gloo rank worker."""

from __future__ import annotations

import os

import numpy as np
import torch

from oracle import packed_ref as ref
from oracle import stack_ref
from tinygrad_dx12_b200 import stack as S
from tinygrad_dx12_b200.packed import PackedTensor

SMALL_INT4 = S.StackConfig(hidden=256, q_dim=256, kv_dim=64, inter=512, layers=2, fmt="int4", block=32, scale="f16u",
                           act=torch.float16)
SMALL_FP4 = S.StackConfig(hidden=256, q_dim=256, kv_dim=64, inter=512, layers=2, fmt="fp4_e2m1", block=32,
                          scale="e8m0", act=torch.bfloat16)
SMALL_FP6 = S.StackConfig(hidden=256, q_dim=256, kv_dim=64, inter=512, layers=2, fmt="fp6_e3m2", block=64,
                          scale="f16u", act=torch.float16)
CONFIGS = {"int4": SMALL_INT4, "fp4": SMALL_FP4, "fp6": SMALL_FP6}
ACT = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


def spec_of(w: PackedTensor) -> ref.PackedSpec:
    data = w.data.cpu().numpy()
    if w.scales is None:
        return ref.PackedSpec(data, w.format, w.shape, None, w.block_size)
    if w.scales.dtype == torch.float8_e8m0fnu:
        e = w.scales.cpu().view(torch.uint8).numpy().astype(np.float64)
        return ref.PackedSpec(data, w.format, w.shape, np.exp2(e - 127).astype(np.float32), w.block_size, "float32")
    return ref.PackedSpec(data, w.format, w.shape, w.scales.cpu().numpy(), w.block_size)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy()


class OracleOps:
    """TPStack compute through the oracle (CPU tensors); the all-reduce through gloo."""

    def linear(self, w, x, out_dtype):
        y = ref.packed_linear_ref(spec_of(w), to_numpy(x))
        return torch.from_numpy(np.ascontiguousarray(y)).to(out_dtype)

    def add_rmsnorm(self, h, partial, x_out):
        h32 = h.float()
        if partial is not None:
            h.copy_((h32 + partial.float()).to(h.dtype))
            h32 = h.float()
        if x_out is not None:
            x_out.copy_(torch.from_numpy(stack_ref.rmsnorm(h32.numpy())).to(x_out.dtype))

    def gate_mul(self, gu, out):
        i = out.shape[1]
        out.copy_((gu[:, :i].float() * gu[:, i:].float()).to(out.dtype))

    def all_reduce(self, t):
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(t)


def full_layers(cfg, device="cpu", seed=0):
    return [{p: S.make_matrix(cfg, layer, p, device, seed) for p in cfg.proj_shapes()} for layer in range(cfg.layers)]


def oracle_forward(cfg, h0: torch.Tensor, seed=0) -> np.ndarray:
    layers = [{p: spec_of(w) for p, w in L.items()} for L in full_layers(cfg, "cpu", seed)]
    return stack_ref.stack_forward(layers, to_numpy(h0), ACT[cfg.act])


def initial_h(cfg, m: int, seed: int = 7) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((m, cfg.hidden), generator=g).to(cfg.act)


def gloo_worker(rank: int, world: int, port: int, cfg_name: str, m: int, out_dir: str) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = CONFIGS[cfg_name]
        st = S.TPStack(cfg, rank, world, device="cpu", ops=OracleOps())
        h = st.forward(initial_h(cfg, m))
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), to_numpy(h))
    finally:
        dist.destroy_process_group()
