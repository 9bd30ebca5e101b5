"""INT4 weight-only layers for a transformers-style model: the public names and signatures of lowbit/model.py of
YuchenHe985/lowbit-kernels (TARGETS, W4Linear, quantize_layers, apply_fake_quant, apply_int4; lowbit/model.py:12-57).

The workflow is the reference's: every decoder projection is quantized once, and the same packed values then back
either a fake-quant model (plain nn.Linear layers holding the dequantized fp16 weights, so torch does the math) or
the INT4 kernels -- a quality gap between the two is kernel error, not quantization error. Here the quantization,
the layouts and the dequantized copies are all built on the GPU, and W4Linear adds its bias inside the kernel's
epilogue instead of with a separate elementwise op.
"""
import torch
from torch import nn

from . import ops

# the projections of a Qwen2 / Llama decoder layer that become INT4 (embeddings and lm_head stay fp16: the head is
# tied to the embedding up to Qwen2.5-3B, so quantizing it would change the embedding too)
TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class W4Linear(nn.Module):
    """A drop-in for nn.Linear over an INT4 weight (lowbit/model.py:15-27): the input is flattened to [M, K] fp16 and
    run through ops.linear -- a decode kernel for few rows, dequantize + cuBLAS for many -- with the bias fused into
    the kernel's epilogue (the same fp16 roundings as adding it to the kernel's output afterwards)."""

    def __init__(self, wq, bias, in_features, out_features, gemv_version=0):
        super().__init__()
        if wq.k != in_features or wq.n != out_features:
            raise ValueError(f"weight is [{wq.n}, {wq.k}], layer is [{out_features}, {in_features}]")
        self.wq = wq
        self.in_features, self.out_features = in_features, out_features
        self.gemv_version = gemv_version
        fp16_bias = None
        if bias is not None:
            fp16_bias = bias.detach().to(device=wq.scales.device, dtype=torch.float16).contiguous()
        # a non-trainable Parameter, as nn.Linear's bias is a Parameter: state_dict and .to() treat it alike
        self.bias = None if fp16_bias is None else nn.Parameter(fp16_bias, requires_grad=False)

    def forward(self, x):
        lead = x.shape[:-1]
        rows = x.reshape(-1, self.in_features)
        if rows.dtype != torch.float16:
            rows = rows.to(torch.float16)
        y = ops.linear(rows, self.wq, version=self.gemv_version,
                       bias=None if self.bias is None else self.bias.data)
        return y.reshape(*lead, self.out_features)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, group={self.wq.group}, "
                f"bias={self.bias is not None}, gemv_version={self.gemv_version}")


def _projections(root):
    """(parent module, attribute name, nn.Linear) for every TARGETS projection under `root`, parents before their
    children, each module visited once."""
    seen = set()

    def walk(parent):
        if id(parent) in seen:
            return
        seen.add(id(parent))
        for name, child in list(parent._modules.items()):
            if child is None:
                continue
            if isinstance(child, nn.Linear) and name in TARGETS:
                yield parent, name, child
            else:
                yield from walk(child)
    yield from walk(root)


def quantize_layers(model, group=128, clip_grid=None):
    """Quantize every decoder projection once, on the GPU (lowbit/model.py:30-39). Returns a list of
    (parent, name, linear, packed, scales): packed uint8 [N, K/2] canonical layout and fp16 scales [N, K/G], both on
    the GPU, bit-identical to lowbit.quant.quantize_w4 at clip_grid=None."""
    return [(parent, name, lin, *ops.quantize_w4_gpu(lin.weight, group, clip_grid))
            for parent, name, lin in _projections(model)]


def apply_fake_quant(layers, group=128):
    """Overwrite each nn.Linear's weight with its dequantized fp16 value: exactly the weights the kernels multiply
    by (lowbit/model.py:42-45)."""
    with torch.no_grad():
        for _, _, lin, packed, scales in layers:
            w16 = ops.dequantize_w4_gpu(packed, scales, group)
            lin.weight.copy_(w16.to(device=lin.weight.device, dtype=lin.weight.dtype))


def apply_int4(layers, group=128, gemv_version=0, layouts=("mma",)):
    """Replace each nn.Linear by a W4Linear over the same packed values, keeping `layouts` of the weight on the GPU
    (no host round trip). Returns (layers replaced, INT4 bytes) and empties `layers`, whose entries held the last
    references to the fp16 projection weights (lowbit/model.py:48-57)."""
    replaced, int4_bytes = 0, 0
    while layers:
        parent, name, lin, packed, scales = layers.pop(0)
        wq = ops.W4Weight(packed, scales, group, layouts)
        setattr(parent, name, W4Linear(wq, lin.bias, lin.in_features, lin.out_features, gemv_version))
        int4_bytes += wq.nbytes()
        replaced += 1
        del lin, packed, scales
    torch.cuda.empty_cache()
    return replaced, int4_bytes
