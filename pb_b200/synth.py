"""Seeded synthetic weights and activations with the shapes and value
distributions the benchmark configurations name (the reference's models and
checkpoints are not available; nibbles are generated directly in the packed
format rather than through quantisation):

  nibbles  uniform 0..15, two per byte, low nibble = even column
  scale    bf16 ~ U(0.004, 0.02) per (row, group)
  bias     bf16 = -8 * scale + N(0, 1e-3)
  router   bf16 ~ N(0, 0.02)
  x        bf16 ~ N(0, 1)

Generation runs on the target device with torch's seeded Philox generator, so
a (seed, shape) pair always yields the same tensors on the same software stack.
"""

from __future__ import annotations

import torch

from . import capi


def gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def q4_scale_bias(rows: int, groups: int, g: torch.Generator, device):
    scale = torch.empty(rows, groups, device=device, dtype=torch.float32).uniform_(0.004, 0.02, generator=g)
    noise = torch.randn(rows, groups, device=device, dtype=torch.float32, generator=g) * 1e-3
    s16 = scale.to(torch.bfloat16)
    b16 = (-8.0 * s16.float() + noise).to(torch.bfloat16)
    return s16, b16


def q4_matrix(rows: int, cols: int, group: int, g: torch.Generator, device):
    """Returns (packed u8 [rows, ceil(cols/2)], scale bf16 [rows, gpr], bias bf16 [rows, gpr])."""
    packed = torch.randint(0, 256, (rows, (cols + 1) // 2), device=device, dtype=torch.uint8, generator=g)
    if cols % 2:
        packed[:, -1] &= 0x0F
    gpr = (cols + group - 1) // group
    s, b = q4_scale_bias(rows, gpr, g, device)
    return packed, s, b


def bf16_bits(t: torch.Tensor) -> torch.Tensor:
    """View a bf16 tensor as its u16 bit patterns (int16 storage)."""
    return t.contiguous().view(torch.int16)


def expert_table(num_experts: int, layout: capi.ExpertLayout, g: torch.Generator, device) -> torch.Tensor:
    """[num_experts, expert_bytes] u8: every slot filled with the fixed-Q4
    component layout (gate/up [I x H], down [H x I])."""
    E, stride = num_experts, int(layout.expert_bytes)
    H, I, G = int(layout.hidden), int(layout.intermediate), int(layout.group_size)
    table = torch.randint(0, 256, (E, stride), device=device, dtype=torch.uint8, generator=g)
    offs = [int(o) for o in layout.component_offsets]
    shapes = [(I, H), (I, H), (H, I)]
    for p, (rows, cols) in enumerate(shapes):
        gpr = cols // G
        s, b = q4_scale_bias(E * rows, gpr, g, device)
        so, bo = offs[3 * p + 1], offs[3 * p + 2]
        nb = rows * gpr * 2
        table[:, so:so + nb] = bf16_bits(s).view(torch.uint8).view(E, nb)
        table[:, bo:bo + nb] = bf16_bits(b).view(torch.uint8).view(E, nb)
    return table


def mxfp4_expert_table(num_experts: int, layout: capi.ExpertLayout, g: torch.Generator, device) -> torch.Tensor:
    """[num_experts, expert_bytes] u8 in the fixed MXFP4 layout: random E2M1
    nibbles, E8M0 scale bytes 119..122 (2^-8..2^-5, weights of magnitude up to
    about 0.2), the zero-sized bias components absent."""
    E, stride = num_experts, int(layout.expert_bytes)
    H, I = int(layout.hidden), int(layout.intermediate)
    table = torch.randint(0, 256, (E, stride), device=device, dtype=torch.uint8, generator=g)
    offs = [int(o) for o in layout.component_offsets]
    for p, (rows, cols) in enumerate([(I, H), (I, H), (H, I)]):
        so, nb = offs[3 * p + 1], rows * (cols // 32)
        table[:, so:so + nb] = torch.randint(119, 123, (E, nb), device=device, dtype=torch.uint8, generator=g)
    return table


def normal_bf16(shape, std: float, g: torch.Generator, device) -> torch.Tensor:
    return (torch.randn(*shape, device=device, dtype=torch.float32, generator=g) * std).to(torch.bfloat16)


def random_routes(tokens: int, num_experts: int, top_k: int, g: torch.Generator, device) -> torch.Tensor:
    """u32-valued int32 [tokens, top_k]: each token's top_k distinct experts,
    uniformly random (the seeded stand-in for a prefill chunk's routing)."""
    keys = torch.rand(tokens, num_experts, device=device, generator=g)
    return keys.topk(top_k, dim=1).indices.to(torch.int32).contiguous()


class MoeLayerWeights:
    """Device-resident weights of one synthetic MoE FFN layer (config 1 shapes
    by default: hidden 2048, 512 experts, intermediate 512, group 64, one
    shared expert with a sigmoid gate)."""

    def __init__(self, device, seed: int, hidden=2048, num_experts=512, intermediate=512, group=64,
                 shared=True, shared_gate=True, mxfp4=False):
        g = gen(device, seed)
        if mxfp4:
            group = 32  # FIXED_MXFP4 slots: one E8M0 scale per 32 columns
        self.hidden, self.num_experts, self.intermediate, self.group = hidden, num_experts, intermediate, group
        self.mxfp4 = mxfp4
        self.layout = (capi.fixed_mxfp4_layout(hidden, intermediate, group) if mxfp4
                       else capi.fixed_q4_layout(hidden, intermediate, group))
        table = mxfp4_expert_table if mxfp4 else expert_table
        self.router = normal_bf16((num_experts, hidden), 0.02, g, device)
        self.experts = table(num_experts, self.layout, g, device)
        self.shared = table(1, self.layout, g, device)[0].contiguous() if shared else None
        self.shared_gate = normal_bf16((hidden,), 0.02, g, device) if (shared and shared_gate) else None

    def c_weights(self) -> capi.MoeWeights:
        ptr = lambda t: None if t is None else t.data_ptr()
        return capi.MoeWeights(self.router.data_ptr(), self.experts.data_ptr(), ptr(self.shared), ptr(self.shared_gate))

    def nbytes(self) -> int:
        return int(self.router.numel() * 2 + self.experts.numel() +
                   (self.shared.numel() if self.shared is not None else 0) +
                   (self.shared_gate.numel() * 2 if self.shared_gate is not None else 0))
