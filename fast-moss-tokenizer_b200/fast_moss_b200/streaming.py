"""Streaming scheduler: CUDA-graph replay with the native v2 attention history.

Keeps the API of fast_moss/streaming.py:28-142 (`StreamingCodec(model)`
entered inside `optimized(model)`, called with (1, 2, samples) FP32 audio,
returning codes, hidden states and the reconstruction; owner thread and
stream rules; history kept at stable addresses).  The scheduling differs:

  * `chunks_per_graph` 80 ms chunks are captured back to back in ONE graph,
    so a file costs ceil(chunks / chunks_per_graph) replays instead of one
    per chunk;
  * every replay writes straight into output buffers allocated once per
    call (one device copy per output per replay), replacing the reference's
    per-chunk clones and the final torch.cat.
"""

from contextlib import ExitStack
from threading import get_ident
from types import MethodType

import torch

from .graphs import GraphedCallable
from .v2_codec import FRAME, _encode_complete
from .v2_runtime import validate


def _stable_cache_update(original):
    def update(module, state, keys, values, positions, *current):
        # Keep the upstream selection and arithmetic, but retain the
        # addresses that the next graph replay reads.
        original(state, keys, values, positions, *current)
        keys.copy_(state.cached_keys)
        values.copy_(state.cached_values)
        positions.copy_(state.cached_positions)
        state.cached_keys = keys
        state.cached_values = values
        state.cached_positions = positions

    return update


class StreamingCodec:
    """Reusable full-file codec for B=1, FP32, 48 kHz stereo CUDA inputs.

    Enter inside ``optimized(model)``.  Each call starts a fresh file and
    preserves native history across 80 ms chunks.
    """

    def __init__(self, model, *, chunks_per_graph=1):
        validate(model)
        if chunks_per_graph < 1:
            raise ValueError("chunks_per_graph must be >= 1")
        self.model = model
        self.device = next(model.parameters()).device
        self.thread = get_ident()
        self.stream = torch.cuda.current_stream(self.device)
        self.chunks_per_graph = int(chunks_per_graph)
        self.stack = None
        self.graph = None
        self.states = []
        self.used = False

    def _check_thread(self):
        if get_ident() != self.thread or torch.cuda.current_stream(self.device) != self.stream:
            raise RuntimeError("Use StreamingCodec on its construction thread and CUDA stream")

    @torch.inference_mode()
    def __enter__(self):
        self._check_thread()
        if self.used:
            raise RuntimeError("Create a new StreamingCodec instead of re-entering")
        if any(getattr(m, "is_streaming", False) for m in self.model.modules()):
            raise RuntimeError("The model already has an active streaming session")
        self.used = True
        self.stack = ExitStack()
        try:
            for module in self.model.modules():
                if not hasattr(module, "_update_streaming_cache"):
                    continue
                if module.context is None:
                    raise ValueError("Streaming graphs require bounded attention history")
                name = "_update_streaming_cache"
                original = getattr(module, name)
                if name in module.__dict__:
                    self.stack.callback(setattr, module, name, module.__dict__[name])
                else:
                    self.stack.callback(delattr, module, name)
                setattr(module, name, MethodType(_stable_cache_update(original), module))
            self.stack.callback(self.model._stop_streaming)
            self.stack.enter_context(self.model.streaming(batch_size=1))
            self.states = [
                m._streaming_state
                for m in self.model.modules()
                if getattr(m, "_streaming_state", None) is not None
            ]
            m = self.chunks_per_graph
            example = torch.zeros(1, 2, FRAME * m, device=self.device)

            def step(audio):
                parts = []
                for i in range(m):
                    chunk = audio[..., i * FRAME:(i + 1) * FRAME]
                    encoded = _encode_complete(self.model, chunk)
                    decoded = self.model._decode_frame(encoded.audio_codes)
                    parts.append((encoded.audio_codes, encoded.encoder_hidden_states,
                                  decoded.audio))
                if m == 1:
                    return parts[0]
                return tuple(torch.cat(p, dim=-1) for p in zip(*parts))

            self.graph = GraphedCallable(step, example)
            self._reset()
            return self
        except BaseException:
            self.__exit__(None, None, None)
            raise

    def _reset(self):
        # Reset contents, never replace storage (graph replays read it).
        for state in self.states:
            state.reset(torch.ones_like(state.exec_mask))

    @torch.inference_mode()
    def __call__(self, audio):
        self._check_thread()
        if self.graph is None:
            raise RuntimeError("Use StreamingCodec inside its active context")
        if (
            audio.ndim != 3
            or audio.shape[:2] != (1, 2)
            or audio.shape[-1] < 1
            or audio.device != self.device
            or audio.dtype != torch.float32
        ):
            raise ValueError("Expected nonempty FP32 CUDA audio with shape (1, 2, samples)")
        self._reset()
        length = audio.shape[-1]
        span = FRAME * self.chunks_per_graph
        padding = (-length) % span
        if padding:
            audio = torch.nn.functional.pad(audio, (0, padding))
        groups = audio.shape[-1] // span
        outputs = None
        for g in range(groups):
            static = self.graph.replay(audio[..., g * span:(g + 1) * span])
            if outputs is None:
                outputs = [torch.empty(t.shape[:-1] + (t.shape[-1] * groups,), device=t.device,
                                       dtype=t.dtype) for t in static]
            for dst, src in zip(outputs, static):
                w = src.shape[-1]
                dst[..., g * w:(g + 1) * w].copy_(src)
        codes, hidden, reconstructed = outputs
        valid = -(-length // FRAME)  # chunks that hold input samples
        frames = codes.shape[-1] // (groups * self.chunks_per_graph) * valid
        hframes = hidden.shape[-1] // (groups * self.chunks_per_graph) * valid
        return codes[..., :frames], hidden[..., :hframes], reconstructed[..., :length]

    def __exit__(self, *exc):
        self._check_thread()
        torch.cuda.synchronize(self.device)
        if self.graph is not None:
            self.graph.release()
        self.graph = None
        self.states = []
        if self.stack is not None:
            self.stack.close()
            self.stack = None
