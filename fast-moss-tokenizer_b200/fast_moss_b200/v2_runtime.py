"""Reversible B200 optimisations of the pinned 48 kHz stereo v2 model.

Drop-in for fast_moss/v2_runtime.py: `optimized(model, cache_linear=True,
quantizer=True, pointwise=True)` replaces the same upstream methods, runs
the B200 path only on the calls the reference's own path covers (every
other call goes to the original method, as in the reference), restores
everything when it closes and keeps the reference's single-owner-thread
rule.

Design.  Each optimisation is one row of PATCHES (a `PatchSpec`): the
modules it applies to, the method it replaces, the `optimized()` switch
that enables it, and a builder.  A builder returns a `_Guarded` method: a
coverage predicate over the call's arguments and the B200 path for the
calls it covers.  The runtime walks the model once on entry, installs the
methods of every matching row as instance attributes, and on exit removes
them in reverse order.  What runs behind the rows:

  transformer layer (reference :231-276): LayerNorm -> attention -> ONE
      kernel for the residual + layer scale + next LayerNorm -> FFN ->
      residual kernel; bit-identical to the reference's scale_add + torch LN;
  rotary embedding (:186-224): ONE kernel computing the phase, cos/sin and
      the rotation (no tables in HBM);
  LFQ decode_latents (:143-181): the reference's prepare + FP32 GEMM +
      select sequence, or (fused_lfq=True) one kernel that never writes the
      [B*T, K] dot-product matrix;
  Linear / weight-norm Conv1d (:77-138): cached bf16 weights and the
      materialised convolution weight (library GEMM / convolution).

Cached resources (bf16 weights, normalised codebooks, conv weights) belong
to the runtime; it holds a `graphs.ResourceLease` for its device while open,
so CUDA graphs captured inside the context stop replaying once it closes.
"""

from collections import Counter
from contextlib import contextmanager
from dataclasses import dataclass
from threading import get_ident
from typing import Callable, Optional

import torch
import torch.nn.functional as F
from torch.nn.modules import module as module_hooks

from . import _lib, graphs
from .v2_loading import REVISION

# Compute capability of the B200 (sm_100) the kernels are built for.
SUPPORTED_CAPABILITY = (10, 0)
_FLOATS = (torch.bfloat16, torch.float32)
_LINEAR_FORWARD = torch.nn.Linear.forward


def validate(model):
    """The pinned 48 kHz stereo checkpoint on an sm_100 device with SDPA
    (the reference's checks, :18-41, with B200 in place of its GPU pin)."""
    if (
        type(model).__name__ != "MossAudioTokenizerModel"
        or getattr(model.config, "_commit_hash", None) != REVISION
        or model.sampling_rate != 48000
        or model.number_channels != 2
        or model.downsample_rate != 3840
        or not model.enable_channel_interleave
    ):
        raise ValueError("Expected the pinned 48 kHz stereo MOSS v2 checkpoint")
    device = next(model.parameters()).device
    if device.type != "cuda":
        raise ValueError("V2 optimizations require CUDA")
    props = torch.cuda.get_device_properties(device)
    if (props.major, props.minor) != SUPPORTED_CAPABILITY:
        raise ValueError("V2 kernels require an sm_100 (B200) GPU")
    if model.attention_implementation != "sdpa":
        raise ValueError("The validated v2 attention backend is SDPA")
    _lib.load()


def _needs_grad(*tensors):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _global_hooks():
    return bool(module_hooks._global_forward_hooks or module_hooks._global_forward_pre_hooks)


def _hooked(module):
    return bool(module._forward_hooks or module._forward_pre_hooks)


def _class_method(module, name):
    """True while `module.<name>` is still its class's own method."""
    return getattr(getattr(module, name), "__func__", None) is getattr(type(module), name)


def _stock_norm(norm, x):
    """A hook-free stock LayerNorm over x's last dimension whose torch CUDA
    forward is the vectorised path the kernels reproduce bit for bit."""
    if type(norm) is not torch.nn.LayerNorm or _hooked(norm):
        return False
    if tuple(norm.normalized_shape) != (x.shape[-1],) or x.shape[-1] % 4:
        return False
    return all(p is None or (p.dtype == torch.float32 and p.device == x.device
                             and p.is_contiguous() and p.data_ptr() % 16 == 0)
               for p in (norm.weight, norm.bias))


class _Guarded:
    """A replacement method: calls that `covers(*args, **kwargs)` accepts
    take `fast`, all others the module's original method."""

    def __init__(self, runtime, original, covers, fast):
        self.runtime = runtime
        self.original = original
        self.covers = covers
        self.fast = fast

    def __call__(self, *args, **kwargs):
        self.runtime._check()
        if self.covers(*args, **kwargs):
            return self.fast(*args, **kwargs)
        return self.original(*args, **kwargs)


# ------------------------------------------------------------ patch builders
def _build_linear(rt, module, original):
    weight, bias = module.weight, module.bias
    versions = (weight._version, None if bias is None else bias._version)
    w16 = weight.to(torch.bfloat16)
    b16 = None if bias is None else bias.to(torch.bfloat16)
    rt.counts["cached_bytes"] += w16.numel() * 2 + (0 if b16 is None else b16.numel() * 2)

    def covers(x):
        return (module.weight is weight and module.bias is bias
                and (weight._version, None if bias is None else bias._version) == versions
                and x.device == rt.device and x.dtype in _FLOATS
                and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and not _needs_grad(x, weight, bias))

    def fast(x):
        rt.counts["linear_calls"] += 1
        return F.linear(x, w16, b16)

    return _Guarded(rt, original, covers, fast)


def _build_conv(rt, module, original):
    weight = module.weight.detach()  # the parametrisation, evaluated once
    params = tuple(module.parametrizations.weight.parameters())
    versions = tuple(p._version for p in params)
    rt.counts["cached_bytes"] += weight.numel() * weight.element_size()

    def covers(x):
        if not torch.nn.utils.parametrize.is_parametrized(module, "weight"):
            return False
        now = tuple(module.parametrizations.weight.parameters())
        return (len(now) == len(params) and all(a is b for a, b in zip(now, params))
                and tuple(p._version for p in params) == versions
                and not _global_hooks()
                and not any(_hooked(m) for m in module.parametrizations.modules())
                and not _needs_grad(x, *params))

    def fast(x):
        return module._conv_forward(x, weight, module.bias)

    return _Guarded(rt, original, covers, fast)


def _build_lfq(rt, module, original):
    from .quantizer import decode_latents, select
    from .quantizer_prepare import prepare

    weight = module.codebook.weight
    version = weight._version
    book = F.normalize(weight.float())  # normalised once, as the reference does
    code_norm = book.pow(2).sum(1, keepdim=True).T
    rt.counts["cached_bytes"] += book.numel() * 4 + code_norm.numel() * 4

    def covers(x):
        return (module.codebook.weight is weight and weight._version == version
                and x.ndim == 3 and x.shape[1] == 8 and x.shape[0] >= 1 and x.shape[2] >= 1
                and x.device == rt.device and x.dtype == torch.float32
                and not torch.is_autocast_enabled("cuda") and not _needs_grad(x, weight))

    def fast(x):
        if x.is_contiguous() and x.numel() < 2 ** 31:
            if rt.fused_lfq:
                rt.counts["select_calls"] += 1
                return decode_latents(x, book, code_norm, weight)
            _, row_norm, twice, _ = prepare(x)
            rt.counts["prepare_calls"] += 1
        else:  # other layouts: the reference's eager normalisation
            latent = F.normalize(x.transpose(1, 2).reshape(-1, 8).float())
            row_norm = latent.pow(2).sum(1, keepdim=True)
            twice = 2 * latent
        rt.counts["select_calls"] += 1
        return select(twice @ book.T, row_norm, code_norm, weight, x)

    return _Guarded(rt, original, covers, fast)


def _build_rotary(rt, module, original):
    from .v2_pointwise import rope

    period = module.max_period

    def covers(q, k, offset, time_before_heads=False):
        return (not time_before_heads and q.ndim == 4 and q.shape == k.shape
                and q.shape[-1] >= 2 and q.shape[-1] % 2 == 0
                and q.dtype in _FLOATS and k.dtype == q.dtype
                and q.device == rt.device and k.device == rt.device
                and offset.device == rt.device and offset.numel() == q.shape[0]
                and module.max_period == period and not _needs_grad(q, k, offset))

    def fast(q, k, offset, time_before_heads=False):
        rt.counts["rope_calls"] += 1
        return rope(q, k, offset.reshape(-1), period)

    return _Guarded(rt, original, covers, fast)


def _build_layer(rt, module, original):
    from .v2_pointwise import layer_norm, residual_layer_norm, scale_add

    scales = (module.layer_scale_1, module.layer_scale_2)
    scale_forwards = tuple(type(s).forward for s in scales)

    def covers(x, **kwargs):
        if (torch.is_grad_enabled() or x.device != rt.device or x.dtype not in _FLOATS
                or module.layer_scale_1 is not scales[0]
                or module.layer_scale_2 is not scales[1] or _global_hooks()):
            return False
        return all(not _hooked(s) and s.channel_last
                   and getattr(s.forward, "__func__", None) is fn
                   and s.scale.dtype == torch.float32 and s.scale.device == rt.device
                   for s, fn in zip(scales, scale_forwards))

    def norm(norm_module, x):
        if x.dtype == torch.float32 and x.is_cuda and _stock_norm(norm_module, x):
            try:
                out = layer_norm(x, norm_module.weight, norm_module.bias, norm_module.eps)
                rt.counts["norm_calls"] += 1
                return out
            except _lib.UnsupportedError:
                pass
        return norm_module(x)

    def kernel_residual(normed, residual, update, scale):
        return (normed.dtype == torch.float32 and update.dtype in _FLOATS
                and residual.shape == update.shape and scale.scale.shape == (residual.shape[-1],)
                and residual.is_contiguous() and update.is_contiguous()
                and scale.scale.is_contiguous())

    def fast(x, **kwargs):
        # attention half; its residual update fused with the next LayerNorm
        normed = norm(module.norm1, x)
        update = module.self_attn(normed, **kwargs)
        normed2 = None
        if kernel_residual(normed, x, update, scales[0]):
            if _stock_norm(module.norm2, x):
                try:
                    x_next, normed2 = residual_layer_norm(
                        x, update, scales[0].scale, module.norm2.weight, module.norm2.bias,
                        module.norm2.eps)
                    rt.counts["fused_norm_calls"] += 1
                except _lib.UnsupportedError:
                    normed2 = None
            if normed2 is None:
                x_next = scale_add(x, update, scales[0].scale)
            rt.counts["residual_calls"] += 1
        else:  # the reference's eager form
            x_next = x.to(normed) + scales[0](update)
        x = x_next
        # feed-forward half
        if normed2 is None:
            normed2 = norm(module.norm2, x)
        update = module.ffn(normed2)
        if kernel_residual(normed2, x, update, scales[1]):
            rt.counts["residual_calls"] += 1
            return scale_add(x, update, scales[1].scale)
        return x.to(normed2) + scales[1](update)

    return _Guarded(rt, original, covers, fast)


# ------------------------------------------------------------ the patch table
@dataclass(frozen=True)
class PatchSpec:
    """One optimisation: `matches(module)` selects the modules, `method` is
    the attribute replaced, `option` the optimized() switch that enables it
    (None: always on), `build(runtime, module, original)` the replacement."""

    key: str
    method: str
    option: Optional[str]
    matches: Callable[[torch.nn.Module], bool]
    build: Callable


def _is_rotary(m):
    return type(m).__name__ == "MossAudioTokenizerRotaryEmbedding"


def _is_layer(m):
    return (type(m).__name__ == "MossAudioTokenizerTransformerLayer"
            and type(m.norm1) is torch.nn.LayerNorm and type(m.norm2) is torch.nn.LayerNorm
            and all(type(s).__name__ == "MossAudioTokenizerLayerScale"
                    for s in (m.layer_scale_1, m.layer_scale_2)))


def _is_linear(m):
    return type(m) is torch.nn.Linear and torch.nn.Linear.forward is _LINEAR_FORWARD


def _is_weight_norm_conv(m):
    return (isinstance(m, torch.nn.Conv1d)
            and torch.nn.utils.parametrize.is_parametrized(m, "weight")
            and getattr(m.forward, "__func__", None) is torch.nn.Conv1d.forward)


def _is_lfq(m):
    return type(m).__name__ == "MossAudioTokenizerLFQ"


PATCHES = (
    PatchSpec("rope", "forward", "pointwise", _is_rotary, _build_rotary),
    PatchSpec("residual", "forward", "pointwise", _is_layer, _build_layer),
    PatchSpec("linear", "forward", "cache_linear", _is_linear, _build_linear),
    PatchSpec("conv", "forward", None, _is_weight_norm_conv, _build_conv),
    PatchSpec("quantizer", "decode_latents", "quantizer", _is_lfq, _build_lfq),
)


class V2Runtime:
    """The optimisation context of one model: single host thread, original
    FP32 parameters left in place.  Counters: `<key>_modules` per patch
    row, `*_calls` per B200 path taken, `cached_bytes`."""

    def __init__(self, model, *, cache_linear=True, quantizer=True, pointwise=True,
                 fused_lfq=False):
        validate(model)
        self.model = model
        self.device = next(model.parameters()).device
        self.thread = get_ident()
        self.options = {"cache_linear": cache_linear, "quantizer": quantizer,
                        "pointwise": pointwise}
        self.fused_lfq = fused_lfq
        self.counts = Counter()
        self.active = self.used = False
        self.lease = None
        self._installed = []  # (module, method, previous own attribute or None)

    def __getattr__(self, name):
        counts = self.__dict__.get("counts")
        if counts is not None and (name.endswith(("_calls", "_modules"))
                                   or name == "cached_bytes"):
            return counts[name]
        raise AttributeError(name)

    def _check(self):
        if not self.active or get_ident() != self.thread:
            raise RuntimeError("Use v2 optimizations on their active owner thread")

    def _admit(self):
        if (self.used or getattr(self.model, "_fast_v2_runtime", None) is not None
                or getattr(self.model, "_fast_optimization_active", False)):
            raise RuntimeError("V2 optimization context is already active or has been used")
        if get_ident() != self.thread:
            raise RuntimeError("Enter v2 optimization on its construction host thread")
        if self.model.training or any(p.requires_grad or p.dtype != torch.float32
                                      or p.device != self.device
                                      for p in self.model.parameters()):
            raise ValueError("V2 optimizations require a frozen FP32 checkpoint on one CUDA device")
        if any(getattr(m, "is_streaming", False) for m in self.model.modules()):
            raise RuntimeError("Enter v2 optimization before starting streaming")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Enter v2 optimization before CUDA graph capture")

    def __enter__(self):
        with torch.cuda.device(self.device):
            self._admit()
            torch.cuda.synchronize(self.device)
        self.lease = graphs.open_lease(self.device, self)
        self.active = self.used = True
        self.model._fast_v2_runtime = self
        try:
            with torch.inference_mode(), torch.autocast("cuda", enabled=False):
                for module in self.model.modules():
                    self._install(module)
        except BaseException:
            self.close()
            raise
        return self

    def _install(self, module):
        for spec in PATCHES:
            if spec.option is not None and not self.options[spec.option]:
                continue
            if not spec.matches(module) or not _class_method(module, spec.method):
                continue
            original = getattr(module, spec.method)
            replacement = spec.build(self, module, original)
            self._installed.append((module, spec.method, module.__dict__.get(spec.method)))
            setattr(module, spec.method, replacement)
            self.counts[f"{spec.key}_modules"] += 1

    def close(self):
        if not self.active:
            return
        try:
            torch.cuda.synchronize(self.device)
        finally:
            if self.lease is not None:
                graphs.close_lease(self.lease)
            for module, method, previous in reversed(self._installed):
                if previous is None:
                    module.__dict__.pop(method, None)
                else:
                    setattr(module, method, previous)
            self._installed.clear()
            self.model.__dict__.pop("_fast_v2_runtime", None)
            self.active = False

    def __exit__(self, *exc):
        self.close()


@contextmanager
def optimized(model, *, cache_linear=True, quantizer=True, pointwise=True, fused_lfq=False):
    """Runs the model's hot path on the B200 kernels inside the context
    (reference fast_moss/v2_runtime.py:441-447)."""
    with V2Runtime(model, cache_linear=cache_linear, quantizer=quantizer, pointwise=pointwise,
                   fused_lfq=fused_lfq) as runtime:
        yield runtime
