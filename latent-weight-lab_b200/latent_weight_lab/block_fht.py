"""BlockFHT generator and BlockFHTLinear -- drop-in API over the sm_100a library.

Public names, signatures, defaults, parameter names (``generator.latent``,
``bias``, ``output_gain``, ...) and ValueError messages follow the reference
module latent_weight_lab/block_fht.py so that state dicts and call sites
interchange.  Differences, by design:

* Every generator evaluation runs in liblwl_b200 kernels on the tensor's GPU,
  for fp32, bf16 and fp16 alike (the reference uses CUDA for fp32 only and
  falls back to a pure-torch loop otherwise, block_fht.py:161,221).
* There is no CPU path: CPU tensors raise instead of silently running a
  different implementation.  The reference's pure-torch oracle
  (block_fht_slice_torch) lives in the test oracle, not here.
* bf16/fp16 math is fp32-accurate or tensor-core factored (see
  ``exact_arithmetic``); results are compared against fp32 math on the same
  rounded latent, not against the reference's stage-by-stage bf16 rounding.
"""
from __future__ import annotations

import contextlib
import math
import threading

import torch
import torch.nn.functional as F
from torch import nn

from . import _native

_STATE = threading.local()


def _flags() -> int:
    return _native.FLAG_EXACT if getattr(_STATE, "exact", False) else 0


@contextlib.contextmanager
def exact_arithmetic(enabled: bool = True):
    """Within this context bf16/fp16 generators use fp32 arithmetic end to end."""
    prev = getattr(_STATE, "exact", False)
    _STATE.exact = bool(enabled)
    try:
        yield
    finally:
        _STATE.exact = prev


def next_power_of_two(value: int) -> int:
    """Smallest power of two >= value (block_fht.py:12-15)."""
    if value <= 0:
        raise ValueError("value must be positive")
    return 1 << (int(value) - 1).bit_length()


def lowbias32(x: int) -> int:
    """32-bit integer finaliser used by the sign hash (block_fht.py:36-43)."""
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return x


def sign_word_for(seed: int, block: int, layer: int, word: int) -> int:
    """The 32 signs of positions 32*word .. 32*word+31 (block_fht.py:46-52)."""
    mask = 0xFFFFFFFF
    x = (int(seed) ^ (int(seed) >> 32)) & mask
    x ^= (0x9E3779B9 * (int(block) + 1)) & mask
    x ^= (0x85EBCA6B * (int(layer) + 1)) & mask
    x ^= (0xC2B2AE35 * (int(word) + 1)) & mask
    return lowbias32(x)


def signs_for(reference: torch.Tensor, block: int, layer: int, seed: int, block_size: int) -> torch.Tensor:
    """+-1 signs of one block/layer as reference's dtype and device (block_fht.py:55-81).

    The words come from the GPU sign kernel; ``reference`` must be a CUDA tensor.
    """
    _native._require_cuda(reference, "reference")
    nwords = (int(block_size) + 31) // 32
    words = _native.sign_words(seed, block, layer, 0, nwords, device=reference.device)
    bits = (words.unsqueeze(1) >> torch.arange(32, device=reference.device)) & 1
    return (2.0 * bits.reshape(-1)[: int(block_size)] - 1.0).to(dtype=reference.dtype)


def _check_slice(start: int, stop: int, size: int) -> None:
    if not 0 <= start <= stop <= size:
        raise ValueError(f"invalid slice [{start}, {stop}) for size {size}")


class _BlockFHTSliceFn(torch.autograd.Function):
    """Autograd over the native forward/backward (block_fht.py:149-196)."""

    @staticmethod
    def forward(ctx, latent, size, layers, seed, start, stop):
        _check_slice(start, stop, size)
        ctx.latent_size = latent.numel()
        ctx.args = (int(size), int(layers), int(seed), int(start), int(stop))
        ctx.flags = _flags()
        return _native.fht_forward(latent.detach(), size, layers, seed, start, stop, flags=ctx.flags)

    @staticmethod
    def backward(ctx, grad_out):
        size, layers, seed, start, stop = ctx.args
        grad = _native.fht_backward(grad_out.contiguous(), ctx.latent_size, size, layers, seed, start, stop,
                                    flags=ctx.flags)
        return grad, None, None, None, None, None


def block_fht_slice(latent: torch.Tensor, size: int, layers: int, seed: int, start: int, stop: int) -> torch.Tensor:
    """Coordinates [start, stop) of the generated vector, differentiable in latent (block_fht.py:199-207)."""
    return _BlockFHTSliceFn.apply(latent, int(size), int(layers), int(seed), int(start), int(stop))


def block_fht_grad_latent(latent: torch.Tensor, grad_out: torch.Tensor, size: int, layers: int, seed: int,
                          start: int = 0, stop: int | None = None) -> torch.Tensor:
    """Vector-Jacobian product of block_fht_slice w.r.t. the latent (block_fht.py:210-248).

    grad_out is cast to the latent dtype first, as in the reference.
    """
    stop = int(size) if stop is None else int(stop)
    _check_slice(int(start), stop, int(size))
    grad_out = grad_out.contiguous().to(dtype=latent.dtype)
    return _native.fht_backward(grad_out, latent.numel(), int(size), int(layers), int(seed), int(start), stop,
                                flags=_flags())


def _generated_weight(latent: torch.Tensor, in_features: int, out_features: int, layers: int, seed: int,
                      weight_scale: float) -> torch.Tensor:
    size = int(in_features) * int(out_features)
    w = _native.fht_forward(latent.detach(), size, layers, seed, 0, size, flags=_flags())
    if float(weight_scale) != 1.0:
        w.mul_(float(weight_scale))
    return w.view(int(out_features), int(in_features))


def block_fht_linear_forward(input: torch.Tensor, latent: torch.Tensor, out_features: int, layers: int, seed: int,
                             weight_scale: float = 1.0) -> torch.Tensor:
    """y = input @ (weight_scale * W)^T with W generated from latent, no autograd (block_fht.py:251-288).

    Like the reference, which takes its fused extension kernel when the shape
    allows it (block_fht.py:263-281), bf16 inputs with in_features % 64 == 0,
    in_features <= 768 and out_features % 128 == 0 run the fused tcgen05
    kernel: each CTA regenerates its weight panel on chip and W never exists in
    device memory.  Other shapes, dtypes and exact_arithmetic() generate W and
    use a library GEMM.
    """
    if input.dim() < 2:
        raise ValueError("input must have at least 2 dimensions")
    in_features = input.shape[-1]
    flat = input.reshape(-1, in_features)
    with torch.no_grad():
        if (flat.is_cuda and flat.dtype == torch.bfloat16 and latent.dtype == torch.bfloat16 and flat.shape[0] > 0
                and not _flags()):
            out = _native.linear_forward(flat, latent, int(out_features), int(layers), int(seed), float(weight_scale))
            if out is not None:
                return out.reshape(*input.shape[:-1], int(out_features))
        w = _generated_weight(latent, in_features, out_features, layers, seed, weight_scale)
        out = F.linear(flat, w.to(dtype=flat.dtype))
    return out.reshape(*input.shape[:-1], int(out_features))


_SIDE_STREAMS: dict = {}


def _side_stream(device: torch.device) -> "torch.cuda.Stream":
    """One extra CUDA stream per device for work that overlaps the caller's stream."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    st = _SIDE_STREAMS.get(key)
    if st is None:
        st = _SIDE_STREAMS[key] = torch.cuda.Stream(device=key)
    return st


class _BlockFHTLinearFn(torch.autograd.Function):
    """Linear layer whose weight is regenerated from the latent (block_fht.py:291-356)."""

    @staticmethod
    def forward(ctx, input, latent, bias, in_features, out_features, size, layers, seed, weight_scale,
                modulation_alpha):
        with torch.no_grad():
            w = _native.fht_forward(latent.detach(), size, layers, seed, 0, size, flags=_flags())
            if float(weight_scale) != 1.0:
                w = w * float(weight_scale)
            if float(modulation_alpha) != 0.0:
                w = w + float(modulation_alpha) * latent.detach().square().sum()
            weight = w.view(int(out_features), int(in_features)).to(dtype=input.dtype)
            output = F.linear(input, weight, bias)
        # The reference regenerates W in backward to save memory (block_fht.py:330-337).
        # W is small next to the activations here, so it is kept for grad_input.
        ctx.save_for_backward(input, latent, weight)
        ctx.has_bias = bias is not None
        ctx.dims = (int(in_features), int(out_features), int(size), int(layers), int(seed))
        ctx.weight_scale = float(weight_scale)
        ctx.modulation_alpha = float(modulation_alpha)
        ctx.flags = _flags()
        return output

    @staticmethod
    def backward(ctx, grad_output):
        input, latent, weight = ctx.saved_tensors
        in_features, out_features, size, layers, seed = ctx.dims
        grad_input = grad_latent = grad_bias = None
        g2 = grad_output.reshape(-1, out_features)
        x2 = input.reshape(-1, in_features)

        def project(grad_weight):
            gl = _native.fht_backward(grad_weight.reshape(-1), latent.numel(), size, layers, seed, 0, size,
                                      flags=ctx.flags)
            if ctx.weight_scale != 1.0:
                gl = gl * ctx.weight_scale
            if ctx.modulation_alpha != 0.0:
                gl = gl + 2.0 * ctx.modulation_alpha * latent * grad_weight.sum()
            return gl

        if ctx.needs_input_grad[1]:
            grad_weight = g2.transpose(0, 1).to(dtype=latent.dtype).matmul(x2.to(dtype=latent.dtype))
            if ctx.needs_input_grad[0]:
                # The latent projection (a few dozen CTAs at GPT widths) and the
                # grad_input GEMM are independent: the projection runs on a side
                # stream, forked after grad_W and joined before returning.
                main = torch.cuda.current_stream(grad_weight.device)
                side = _side_stream(grad_weight.device)
                side.wait_stream(main)
                with torch.cuda.stream(side):
                    grad_latent = project(grad_weight)
                grad_weight.record_stream(side)
                grad_input = g2.matmul(weight.to(dtype=grad_output.dtype)).reshape_as(input)
                main.wait_stream(side)
                grad_latent.record_stream(main)
            else:
                grad_latent = project(grad_weight)
        elif ctx.needs_input_grad[0]:
            grad_input = g2.matmul(weight.to(dtype=grad_output.dtype)).reshape_as(input)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            grad_bias = g2.sum(dim=0).to(dtype=grad_output.dtype)
        return grad_input, grad_latent, grad_bias, None, None, None, None, None, None, None


class BlockFHTLinear(nn.Module):
    """nn.Linear replacement whose [out, in] weight is a BlockFHT of a small latent.

    Constructor, parameters and buffers follow block_fht.py:359-425.  The
    optional extras (modulation, residual base, gains, spectral correction)
    are composed with torch ops on the generated weight exactly as the
    reference composes them (block_fht.py:437-462).
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        bias: bool = False,
        latent_dim: int | None = None,
        latent_ratio: float = 0.01,
        layers: int = 3,
        seed: int = 0,
        latent_init_std: float = 0.02,
        weight_scale: float = 1.0,
        modulation_alpha: float = 0.0,
        modulation_centered: bool = False,
        residual_base_scale: float = 0.0,
        residual_base_std: float = 0.02,
        output_gain: bool = False,
        input_gain: bool = False,
        spectral_rank: int = 0,
        spectral_out_groups: int = 1,
        spectral_in_groups: int = 1,
    ) -> None:
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        size = self.in_features * self.out_features
        if latent_dim is None:
            latent_dim = max(1, round(size * float(latent_ratio)))
        self.generator = BlockFHT(int(latent_dim), size=size, layers=layers, seed=seed,
                                  latent_init_std=latent_init_std)
        self.bias = nn.Parameter(torch.zeros(self.out_features)) if bias else None
        self._cached_weight: torch.Tensor | None = None
        self.weight_scale = float(weight_scale)
        self.modulation_alpha = float(modulation_alpha)
        self.modulation_centered = bool(modulation_centered)
        self.latent_init_std = float(latent_init_std)
        self.residual_base_scale = float(residual_base_scale)
        self.output_gain = nn.Parameter(torch.ones(self.out_features)) if output_gain else None
        self.input_gain = nn.Parameter(torch.ones(self.in_features)) if input_gain else None
        self.spectral_rank = int(spectral_rank)
        self.spectral_out_groups = int(spectral_out_groups)
        self.spectral_in_groups = int(spectral_in_groups)
        if self.spectral_rank:
            if self.spectral_rank > min(self.in_features, self.out_features):
                raise ValueError("spectral_rank exceeds matrix dimensions")
            if self.out_features % self.spectral_out_groups or self.in_features % self.spectral_in_groups:
                raise ValueError("spectral gain groups must divide feature dimensions")
            self.register_buffer("spectral_u", self._hadamard_columns(self.out_features, self.spectral_rank, seed + 17),
                                 persistent=True)
            self.register_buffer("spectral_v", self._hadamard_columns(self.in_features, self.spectral_rank, seed + 31),
                                 persistent=True)
            self.spectral_core = nn.Parameter(torch.zeros(self.spectral_rank, self.spectral_rank))
            self.spectral_log_out_gain = nn.Parameter(torch.zeros(self.spectral_out_groups))
            self.spectral_log_in_gain = nn.Parameter(torch.zeros(self.spectral_in_groups))
        else:
            self.spectral_u = self.spectral_v = None
            self.spectral_core = self.spectral_log_out_gain = self.spectral_log_in_gain = None
        if self.residual_base_scale != 0.0:
            base = torch.empty(self.out_features, self.in_features)
            nn.init.normal_(base, mean=0.0, std=float(residual_base_std))
            self.register_buffer("residual_base_weight", base, persistent=True)
        else:
            self.residual_base_weight = None

    @staticmethod
    def _hadamard_columns(length: int, rank: int, seed: int) -> torch.Tensor:
        """Columns seed..seed+rank-1 of the natural-order Hadamard matrix, / sqrt(length)."""
        rows = torch.arange(length, dtype=torch.int64).view(-1, 1)
        cols = (torch.arange(rank, dtype=torch.int64) + int(seed)).view(1, -1)
        bits = rows.bitwise_and(cols)
        parity = torch.zeros_like(bits)
        while bits.any():
            parity = parity.bitwise_xor(bits.bitwise_and(1))
            bits = bits.bitwise_right_shift(1)
        return (1.0 - 2.0 * parity.float()) / math.sqrt(length)

    def _modulation_offset(self) -> torch.Tensor:
        offset = self.generator.latent.square().sum()
        if self.modulation_centered:
            expected = self.generator.latent.numel() * self.latent_init_std * self.latent_init_std
            offset = offset - offset.new_tensor(expected)
        return offset

    def _has_extras(self) -> bool:
        return (self.residual_base_weight is not None or self.modulation_centered or self.output_gain is not None
                or self.input_gain is not None or self.spectral_core is not None)

    @property
    def weight(self) -> torch.Tensor:
        """The effective [out, in] weight, differentiable in every parameter."""
        return self._compose_weight(self.generator())

    def _compose_weight(self, generated: torch.Tensor) -> torch.Tensor:
        """Scale, modulation, residual base, spectral correction and gains around the generated vector."""
        weight = generated * self.weight_scale
        if self.modulation_alpha != 0.0:
            weight = weight + self.modulation_alpha * self._modulation_offset()
        weight = weight.view(self.out_features, self.in_features)
        if self.residual_base_weight is not None:
            weight = self.residual_base_weight.to(device=weight.device, dtype=weight.dtype) + \
                self.residual_base_scale * weight
        if self.spectral_core is not None:
            dt = weight.dtype
            correction = self.spectral_u.to(dtype=dt).matmul(self.spectral_core.to(dtype=dt)).matmul(
                self.spectral_v.to(dtype=dt).transpose(0, 1))
            weight = weight + correction
            out_gain = self.spectral_log_out_gain.exp().repeat_interleave(
                self.out_features // self.spectral_out_groups).to(dtype=dt)
            in_gain = self.spectral_log_in_gain.exp().repeat_interleave(
                self.in_features // self.spectral_in_groups).to(dtype=dt)
            weight = weight * out_gain.view(-1, 1) * in_gain.view(1, -1)
        if self.output_gain is not None:
            weight = weight * self.output_gain.to(device=weight.device, dtype=weight.dtype).view(-1, 1)
        if self.input_gain is not None:
            weight = weight * self.input_gain.to(device=weight.device, dtype=weight.dtype).view(1, -1)
        return weight

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if self._cached_weight is not None:
            return F.linear(input, self._cached_weight, self.bias)
        if self._has_extras():
            return F.linear(input, self.weight.to(dtype=input.dtype), self.bias)
        return _BlockFHTLinearFn.apply(input, self.generator.latent, self.bias, self.in_features, self.out_features,
                                       self.generator.size, self.generator.layers, self.generator.seed,
                                       self.weight_scale, self.modulation_alpha)

    def _forward_fused_ex(self, input: torch.Tensor, weight_scale: float) -> torch.Tensor | None:
        # like the reference's materialised path (F.linear with self.weight),
        # the call's weight_scale argument does not enter when gains are set;
        # without gains it scales the generated part, as in block_fht.py:487-494
        gains = self.output_gain is not None or self.input_gain is not None
        scale = self.weight_scale if gains else weight_scale * self.weight_scale
        lat = self.generator.latent
        if not (input.is_cuda and input.dtype == torch.bfloat16 and lat.dtype == torch.bfloat16) or _flags():
            return None
        flat = input.reshape(-1, self.in_features)
        if flat.shape[0] == 0:
            return None
        with torch.no_grad():
            # the modulation term (alpha * offset added to every weight element,
            # block_fht.py:448-449) stays on the device as an fp32 scalar and is
            # added to the generated panel on chip, under the gains like the
            # reference's weight property
            offset = (self.modulation_alpha * self._modulation_offset().float()
                      if self.modulation_alpha != 0.0 else None)
            base = self.residual_base_weight
            out = _native.linear_forward(flat, lat, self.out_features, self.generator.layers, self.generator.seed,
                                         scale, bias=self.bias,
                                         output_gain=self.output_gain, input_gain=self.input_gain,
                                         weight_offset=offset, base=base,
                                         base_scale=self.residual_base_scale if base is not None else 1.0)
            if out is None:
                return None
        return out.reshape(*input.shape[:-1], self.out_features)

    def forward_fused(self, input: torch.Tensor, weight_scale: float = 1.0) -> torch.Tensor:
        """Inference forward without autograd (block_fht.py:482-501).

        With output/input gains the reference multiplies a materialised
        weight, and with a residual base it runs a second GEMM; here, for
        bf16 layers the fused kernel takes, the gains, the modulation offset,
        the residual base and the bias are folded into the on-chip panel and
        the epilogue instead (one GEMM).
        """
        if (self.output_gain is not None or self.input_gain is not None or self.modulation_alpha != 0.0
                or self.residual_base_weight is not None) and self.spectral_core is None:
            out = self._forward_fused_ex(input, weight_scale)
            if out is not None:
                return out
        if self.output_gain is not None or self.input_gain is not None or self.spectral_core is not None:
            return F.linear(input, self.weight.to(dtype=input.dtype), self.bias)
        out = block_fht_linear_forward(input, self.generator.latent, self.out_features, self.generator.layers,
                                       self.generator.seed, weight_scale=weight_scale * self.weight_scale)
        if self.modulation_alpha != 0.0:
            modulation = self.modulation_alpha * self._modulation_offset()
            out = out + modulation.to(dtype=out.dtype) * input.sum(dim=-1, keepdim=True)
        if self.residual_base_weight is not None:
            base_out = F.linear(input, self.residual_base_weight.to(device=input.device, dtype=input.dtype))
            out = base_out + self.residual_base_scale * out
        if self.bias is not None:
            out = out + self.bias
        return out

    def materialize_weight_cache(self, dtype: torch.dtype | None = None) -> None:
        """Generate the weight once as a leaf tensor for several microbatches (block_fht.py:503-512)."""
        if self.residual_base_weight is not None or self.spectral_core is not None:
            return
        if self._cached_weight is not None:
            return
        with torch.no_grad():
            weight = self.weight
            if dtype is not None:
                weight = weight.to(dtype=dtype)
        self._cached_weight = weight.detach().requires_grad_(True)

    def _flush_prepare(self) -> torch.Tensor | None:
        """First half of the cache flush: the gain gradients, and the gradient
        of the generated weight as a flat tensor in the latent dtype (None when
        there is nothing to project)."""
        if self._cached_weight is None or self._cached_weight.grad is None:
            return None
        ldt = self.generator.latent.dtype
        grad_weight = self._cached_weight.grad.to(dtype=ldt)
        cached_weight = self._cached_weight.detach().to(dtype=ldt)
        generated_grad_weight = grad_weight
        if self.output_gain is not None:
            output_gain = self.output_gain.detach().to(dtype=ldt)
            if torch.any(output_gain == 0):
                raise RuntimeError("cannot flush a cached BlockFHT weight with a zero output gain")
            g = (grad_weight * (cached_weight / output_gain.view(-1, 1))).sum(dim=1)
            if self.output_gain.grad is None:
                self.output_gain.grad = g.to(dtype=self.output_gain.dtype)
            else:
                self.output_gain.grad.add_(g.to(dtype=self.output_gain.dtype))
            generated_grad_weight = generated_grad_weight * output_gain.view(-1, 1)
        if self.input_gain is not None:
            input_gain = self.input_gain.detach().to(dtype=ldt)
            if torch.any(input_gain == 0):
                raise RuntimeError("cannot flush a cached BlockFHT weight with a zero input gain")
            g = (grad_weight * (cached_weight / input_gain.view(1, -1))).sum(dim=0)
            if self.input_gain.grad is None:
                self.input_gain.grad = g.to(dtype=self.input_gain.dtype)
            else:
                self.input_gain.grad.add_(g.to(dtype=self.input_gain.dtype))
            generated_grad_weight = generated_grad_weight * input_gain.view(1, -1)
        generated_grad_weight = generated_grad_weight.reshape(-1)
        if self.residual_base_weight is not None:
            generated_grad_weight = generated_grad_weight * self.residual_base_scale
        return generated_grad_weight.contiguous()

    def _flush_finish(self, generated_grad_weight: torch.Tensor, projected: torch.Tensor) -> None:
        """Second half: scale the projected gradient, add the modulation term,
        accumulate into the latent's gradient and drop the cache."""
        grad_latent = self.weight_scale * projected
        if self.modulation_alpha != 0.0:
            # same value as block_fht.py:551-552; the latent is detached so the
            # stored gradient carries no autograd graph
            grad_latent = grad_latent + 2.0 * self.modulation_alpha * self.generator.latent.detach() * \
                generated_grad_weight.sum()
        if self.generator.latent.grad is None:
            self.generator.latent.grad = grad_latent
        else:
            self.generator.latent.grad.add_(grad_latent)
        self._cached_weight = None

    def flush_weight_cache_to_latent_grad(self) -> None:
        """Project the cached weight's gradient onto the latent and gains (block_fht.py:514-557)."""
        if self._cached_weight is None:
            return
        g = self._flush_prepare()
        if g is not None:
            self._flush_finish(g, block_fht_grad_latent(self.generator.latent, g, self.generator.size,
                                                        self.generator.layers, self.generator.seed))
        self._cached_weight = None


def prepare_block_fht_weight_cache(model: nn.Module, dtype: torch.dtype | None = None) -> None:
    """Materialise every BlockFHTLinear weight of `model` (block_fht.py:560-563).

    The generators are run together: one grouped library call per
    (device, dtype) instead of one call per module.
    """
    modules = [m for m in model.modules() if isinstance(m, BlockFHTLinear)]
    todo = [m for m in modules
            if m._cached_weight is None and m.residual_base_weight is None and m.spectral_core is None]
    groups: dict[tuple, list[BlockFHTLinear]] = {}
    for m in todo:
        lat = m.generator.latent
        # the grouped launch serves 16-bit generators with blocks up to 2^15; the rest go one by one
        if lat.is_cuda and lat.dtype in (torch.bfloat16, torch.float16) and m.generator.block_size <= 32768:
            groups.setdefault((lat.device, lat.dtype), []).append(m)
    with torch.no_grad():
        for mods in groups.values():
            raws = _native.fht_forward_grouped(
                [(m.generator.latent, m.generator.size, m.generator.layers, m.generator.seed, 0, m.generator.size)
                 for m in mods], flags=_flags())
            for m, raw in zip(mods, raws):
                weight = m._compose_weight(raw)
                if dtype is not None:
                    weight = weight.to(dtype=dtype)
                m._cached_weight = weight.detach().requires_grad_(True)
    for module in modules:
        module.materialize_weight_cache(dtype=dtype)


def flush_block_fht_weight_cache(model: nn.Module) -> None:
    """Project every cached weight gradient of `model` onto its latent (block_fht.py:566-569).

    The latent projections of CUDA generators run together: one grouped
    library call (lwl_fht_backward_grouped) per (device, dtype).
    """
    pending: dict[tuple, list[tuple[BlockFHTLinear, torch.Tensor]]] = {}
    for module in model.modules():
        if not isinstance(module, BlockFHTLinear) or module._cached_weight is None:
            continue
        lat = module.generator.latent
        if not lat.is_cuda:
            module.flush_weight_cache_to_latent_grad()
            continue
        g = module._flush_prepare()
        if g is None:
            module._cached_weight = None
            continue
        pending.setdefault((lat.device, lat.dtype), []).append((module, g))
    for mods in pending.values():
        projected = _native.fht_backward_grouped(
            [(g, m.generator.latent.numel(), m.generator.size, m.generator.layers, m.generator.seed, 0,
              m.generator.size) for m, g in mods], flags=_flags())
        for (m, g), pz in zip(mods, projected):
            m._flush_finish(g, pz)


def suspend_block_fht_weight_cache(model: nn.Module) -> list[tuple[BlockFHTLinear, torch.Tensor]]:
    """Detach cached weights so a forward sees the live latent; keep them for restore (block_fht.py:572-586)."""
    suspended: list[tuple[BlockFHTLinear, torch.Tensor]] = []
    for module in model.modules():
        if isinstance(module, BlockFHTLinear) and module._cached_weight is not None:
            suspended.append((module, module._cached_weight))
            module._cached_weight = None
    return suspended


def restore_block_fht_weight_cache(suspended: list[tuple[BlockFHTLinear, torch.Tensor]]) -> None:
    """Undo suspend_block_fht_weight_cache (block_fht.py:589-594)."""
    for module, weight in suspended:
        if module._cached_weight is not None:
            raise RuntimeError("cannot restore BlockFHT cache over a live cached weight")
        module._cached_weight = weight


class BlockFHT(nn.Module):
    """Stateless-hash block Hadamard generator of `size` coordinates (block_fht.py:597-641)."""

    def __init__(self, latent: int | torch.Tensor | nn.Parameter, size: int, layers: int = 3, seed: int = 0,
                 latent_init_std: float = 0.02) -> None:
        super().__init__()
        if size <= 0:
            raise ValueError("size must be positive")
        if layers not in {1, 2, 3}:
            raise ValueError("layers must be 1, 2, or 3")
        if isinstance(latent, int):
            if latent <= 0:
                raise ValueError("latent size must be positive")
            self.latent_size = int(latent)
            self.latent = nn.Parameter(torch.empty(self.latent_size))
            nn.init.normal_(self.latent, std=float(latent_init_std))
        else:
            if latent.dim() != 1:
                raise ValueError("latent tensor must be 1D")
            self.latent_size = int(latent.numel())
            self.latent = latent if isinstance(latent, nn.Parameter) else nn.Parameter(latent)
        self.size = int(size)
        self.layers = int(layers)
        self.seed = int(seed)
        self.block_size = next_power_of_two(self.latent_size)

    def extra_repr(self) -> str:
        return (f"latent_size={self.latent_size}, size={self.size}, layers={self.layers}, "
                f"seed={self.seed}, block_size={self.block_size}")

    def slice(self, start: int, stop: int) -> torch.Tensor:
        return block_fht_slice(self.latent, self.size, self.layers, self.seed, start, stop)

    def forward(self) -> torch.Tensor:
        return self.slice(0, self.size)

    @property
    def cuda_extension_error(self) -> Exception | None:
        """Load error of the native library (None when it loaded or was not needed yet)."""
        return _native.load_error()
