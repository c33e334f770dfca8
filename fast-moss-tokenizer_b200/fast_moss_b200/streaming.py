"""StreamingCodec: a batch-1 stereo file encoded and decoded 80 ms at a time
under CUDA graphs.

Drop-in for fast_moss/streaming.py (`StreamingCodec(model)` entered inside
`optimized(model)`, called with (1, 2, samples) FP32 audio on the model's
device, returning codes, encoder hidden states and the reconstruction;
one owner thread and stream).  How it runs:

  * the step (encode + quantize + decode of `chunks_per_graph` frames,
    v2_codec._encode_complete and the model's _decode_frame) is captured
    once as a `graphs.CapturedStep`; each call writes the audio of the next
    frames straight into the step's static input and replays, so a file
    costs ceil(frames / chunks_per_graph) replays;
  * a replay reads the attention history at fixed addresses.  The upstream
    streaming modules rebind new history tensors on every update, so while
    the session is open each module's `_update_streaming_cache` is wrapped
    by `_KeepAddresses`, which moves the new window back into the tensors
    the module held before the update;
  * each replay's outputs are copied once into buffers allocated per call
    (no per-chunk clone, no concatenation).
"""

from threading import get_ident

import torch
import torch.nn.functional as F

from .graphs import CapturedStep
from .v2_codec import FRAME, _encode_complete
from .v2_runtime import validate

_HISTORY = ("cached_keys", "cached_values", "cached_positions")


class _KeepAddresses:
    """Stands in for a streaming module's `_update_streaming_cache`: runs the
    upstream update, then copies every history field it rebound back into
    the tensor that held the field before, and points the field at it
    again."""

    def __init__(self, update):
        self.update = update

    def __call__(self, state, *args):
        held = [getattr(state, name) for name in _HISTORY]
        self.update(state, *args)
        for name, buf in zip(_HISTORY, held):
            new = getattr(state, name)
            if new is not buf:
                buf.copy_(new)
                setattr(state, name, buf)


def _streaming(model):
    return any(getattr(m, "is_streaming", False) for m in model.modules())


class StreamingCodec:
    """Reusable full-file codec for batch-1, FP32, 48 kHz stereo CUDA audio.

    Enter it inside ``optimized(model)``; each call codes one whole file
    from a fresh history, which carries across the file's 80 ms frames.
    Not re-enterable: build a new one for a new session.
    """

    def __init__(self, model, *, chunks_per_graph=1):
        validate(model)
        if chunks_per_graph < 1:
            raise ValueError("chunks_per_graph must be >= 1")
        self.model = model
        self.device = next(model.parameters()).device
        self.owner = (get_ident(), torch.cuda.current_stream(self.device))
        self.chunks_per_graph = int(chunks_per_graph)
        self.span = FRAME * self.chunks_per_graph
        self._undo = None  # restore actions of the open session, in order
        self._step = None
        self._states = []
        self._entered = False

    def _own(self):
        if (get_ident(), torch.cuda.current_stream(self.device)) != self.owner:
            raise RuntimeError("StreamingCodec runs on the host thread and CUDA stream that "
                               "built it")

    # ------------------------------------------------------------- session
    @torch.inference_mode()
    def __enter__(self):
        self._own()
        if self._entered:
            raise RuntimeError("a StreamingCodec session cannot be re-entered; build a new one")
        if _streaming(self.model):
            raise RuntimeError("the model already has a live streaming session")
        self._entered = True
        self._undo = []
        try:
            self._open()
        except BaseException:
            self._close()
            raise
        return self

    def _open(self):
        for module in self.model.modules():
            if not hasattr(module, "_update_streaming_cache"):
                continue
            if module.context is None:
                raise ValueError("graph replay needs a bounded attention history "
                                 "(a streaming module has context=None)")
            own = module.__dict__.get("_update_streaming_cache")
            if own is None:
                self._undo.append(lambda m=module: m.__dict__.pop("_update_streaming_cache",
                                                                  None))
            else:
                self._undo.append(lambda m=module, f=own: setattr(m, "_update_streaming_cache",
                                                                  f))
            module._update_streaming_cache = _KeepAddresses(module._update_streaming_cache)
        # undone in reverse: the session's own exit first, then a stop in
        # case it left the model streaming
        self._undo.append(lambda: self.model._stop_streaming() if _streaming(self.model)
                          else None)
        session = self.model.streaming(batch_size=1)
        session.__enter__()
        self._undo.append(lambda: session.__exit__(None, None, None))
        self._states = [m._streaming_state for m in self.model.modules()
                        if getattr(m, "_streaming_state", None) is not None]
        model, frames = self.model, self.chunks_per_graph

        def step(audio):
            codes, hidden, recon = [], [], []
            for i in range(frames):
                encoded = _encode_complete(model, audio[..., i * FRAME:(i + 1) * FRAME])
                codes.append(encoded.audio_codes)
                hidden.append(encoded.encoder_hidden_states)
                recon.append(model._decode_frame(encoded.audio_codes).audio)
            if frames == 1:
                return codes[0], hidden[0], recon[0]
            return torch.cat(codes, -1), torch.cat(hidden, -1), torch.cat(recon, -1)

        audio = torch.zeros(1, 2, self.span, device=self.device)
        self._step = CapturedStep(step, [audio])
        self._restart()

    def _restart(self):
        """A fresh file: every history reset in place (replays read it)."""
        for state in self._states:
            state.reset(torch.ones_like(state.exec_mask))

    def _close(self):
        if self._step is not None:
            self._step.release()
            self._step = None
        self._states = []
        undo, self._undo = self._undo or [], None
        for action in reversed(undo):
            action()

    def __exit__(self, *exc):
        self._own()
        torch.cuda.synchronize(self.device)
        self._close()

    # ---------------------------------------------------------------- calls
    @torch.inference_mode()
    def __call__(self, audio):
        """Codes one file: audio (1, 2, samples) FP32 on the model's device.
        Returns (codes, encoder hidden states, reconstruction), the last
        trimmed to the input length."""
        self._own()
        if self._step is None:
            raise RuntimeError("call StreamingCodec inside its active context")
        if (audio.ndim != 3 or tuple(audio.shape[:2]) != (1, 2) or audio.shape[-1] < 1
                or audio.device != self.device or audio.dtype != torch.float32):
            raise ValueError("expected nonempty FP32 audio of shape (1, 2, samples) on "
                             f"{self.device}")
        self._restart()
        samples = audio.shape[-1]
        replays = -(-samples // self.span)
        if replays * self.span != samples:
            audio = F.pad(audio, (0, replays * self.span - samples))
        slot = self._step.inputs[0]
        outputs = None
        for r in range(replays):
            slot.copy_(audio[..., r * self.span:(r + 1) * self.span])
            produced = self._step.replay()
            if outputs is None:
                outputs = [torch.empty(t.shape[:-1] + (t.shape[-1] * replays,), device=t.device,
                                       dtype=t.dtype) for t in produced]
            for dst, src in zip(outputs, produced):
                width = src.shape[-1]
                dst[..., r * width:(r + 1) * width].copy_(src)
        codes, hidden, recon = outputs
        frames = -(-samples // FRAME)  # frames that hold input samples
        per_frame_codes = codes.shape[-1] // (replays * self.chunks_per_graph)
        per_frame_hidden = hidden.shape[-1] // (replays * self.chunks_per_graph)
        return (codes[..., :frames * per_frame_codes], hidden[..., :frames * per_frame_hidden],
                recon[..., :samples])
