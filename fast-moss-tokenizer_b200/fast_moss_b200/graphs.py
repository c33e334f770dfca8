"""CUDA graphs for fixed-shape steps, and the validity of what they capture.

`CapturedStep` is the primitive the schedulers of this package replay.  Its
step function reads tensors the step owns (`inputs`) and returns the tensors
it writes (`outputs`); it is warmed up on a side stream, captured once, and
every `replay()` reruns it in place on the stream that built it, without
allocating.  Callers write the next inputs straight into `inputs` (a copy
from pinned host memory can land there directly) and read `outputs` until
the next replay.

A captured step holds raw addresses.  Some of them belong to device
resources that an optimisation context (`v2_runtime.V2Runtime`) builds and
owns: cached bf16 weights, normalised codebooks, precomputed convolution
weights.  Each open context holds a `ResourceLease` on its device; a step
captured while leases are open keeps their stamps and refuses to replay
once any of those contexts has rebuilt or released its resources.  A step
captured with no context open depends on no such resources.

`GraphedCallable(fn, *examples)` keeps the reference's public form
(fast_moss/graphs.py:6-60: capture after a warm-up, calls copy the
arguments into static buffers and return clones the caller owns) on top of
CapturedStep; `replay(*args)` is its allocation-free variant.
"""

import threading

import torch

_LEASES = {}
_LEASES_LOCK = threading.Lock()


class ResourceLease:
    """Validity of the cached device resources of one optimisation context.

    The owner calls `renew()` whenever it rebuilds or drops a resource and
    `revoke()` when it closes.  A holder keeps `stamp()` from the time it
    captured and asks `valid(stamp)` before it uses the addresses again.
    """

    def __init__(self, device, owner):
        self.device = device
        self.owner = owner
        self._generation = 0
        self._revoked = False

    def stamp(self):
        return self._generation

    def renew(self):
        self._generation += 1

    def revoke(self):
        self._revoked = True
        self._generation += 1

    def valid(self, stamp):
        return not self._revoked and stamp == self._generation


def open_lease(device, owner):
    """Registers and returns a new lease of `owner` on `device`."""
    lease = ResourceLease(torch.device(device), owner)
    with _LEASES_LOCK:
        _LEASES.setdefault(lease.device, []).append(lease)
    return lease


def close_lease(lease):
    """Revokes `lease` and unregisters it from its device."""
    with _LEASES_LOCK:
        lease.revoke()
        held = _LEASES.get(lease.device, [])
        if lease in held:
            held.remove(lease)


def current_leases(device):
    """The leases of the contexts open on `device` (a tuple, maybe empty)."""
    with _LEASES_LOCK:
        return tuple(_LEASES.get(torch.device(device), ()))


class CapturedStep:
    """`fn(*inputs)` captured once into a CUDA graph and replayed in place.

    inputs: CUDA tensors on one device that the step owns from now on (the
    caller refills them between replays).  fn must return a tuple of
    tensors; those become `outputs`, overwritten by every replay.
    """

    @torch.inference_mode()
    def __init__(self, fn, inputs, *, warmup=3):
        inputs = tuple(inputs)
        if not inputs or not all(isinstance(t, torch.Tensor) and t.is_cuda for t in inputs):
            raise ValueError("CUDA tensor examples required")
        self.device = inputs[0].device
        if any(t.device != self.device for t in inputs):
            raise ValueError("All graph inputs must be on one device")
        self.inputs = inputs
        self.stream = torch.cuda.current_stream(self.device)
        leases = current_leases(self.device)
        stamps = tuple(lease.stamp() for lease in leases)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*inputs)
        self.stream.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            outputs = fn(*inputs)
        self.stream.wait_stream(side)
        if current_leases(self.device) != leases or not self._leases_valid(leases, stamps):
            self.graph = None
            raise RuntimeError("An optimisation context opened, closed or rebuilt its cached "
                               "resources during graph construction; build the graph inside "
                               "one active context")
        if not isinstance(outputs, tuple) or not all(isinstance(t, torch.Tensor)
                                                     for t in outputs):
            self.graph = None
            raise TypeError("Captured function must return a tuple of tensors")
        self.outputs = outputs
        self.leases, self.stamps = leases, stamps

    @staticmethod
    def _leases_valid(leases, stamps):
        return all(lease.valid(stamp) for lease, stamp in zip(leases, stamps))

    def _ready(self):
        if self.graph is None:
            raise RuntimeError("This captured step has been released")
        if not self._leases_valid(self.leases, self.stamps):
            raise RuntimeError("The cached resources this graph captured were released or "
                               "rebuilt; construct a new graph in the active context")
        if torch.cuda.current_stream(self.device) != self.stream:
            raise RuntimeError("Replay this graph on the stream that constructed it")

    def replay(self):
        """Reruns the step on the current inputs; returns `outputs`."""
        self._ready()
        self.graph.replay()
        return self.outputs

    def release(self):
        """Drops the graph and the step's buffers."""
        self.graph = None
        self.outputs = None
        self.inputs = None


class GraphedCallable:
    """`fn` captured after a warm-up on a side stream (reference form).

    Calls run on the CUDA stream used during construction, copy their
    arguments into the static inputs and return clones owned by the caller;
    `replay(*args)` returns the static outputs themselves (valid until the
    next replay).  A graph built inside an optimisation context stops
    working when the context closes or rebuilds its cached resources.
    """

    def __init__(self, fn, *examples, warmup=3):
        if not examples:
            raise ValueError("CUDA tensor examples required")
        self._step = CapturedStep(fn, [t.clone() for t in examples], warmup=warmup)
        self.device = self._step.device

    @property
    def inputs(self):
        return self._step.inputs

    @property
    def outputs(self):
        return self._step.outputs

    @torch.inference_mode()
    def replay(self, *args):
        """Copies args into the static inputs, replays, returns the static
        outputs (overwritten by the next replay)."""
        inputs = self._step.inputs
        if inputs is None:
            raise RuntimeError("This captured step has been released")
        if len(args) != len(inputs):
            raise ValueError("Input count differs from capture")
        for src, dst in zip(args, inputs):
            if (src.shape, src.dtype, src.device) != (dst.shape, dst.dtype, dst.device):
                raise ValueError("Input shape, dtype, and device must match capture")
        self._step._ready()
        for src, dst in zip(args, inputs):
            dst.copy_(src)
        return self._step.replay()

    @torch.inference_mode()
    def __call__(self, *args):
        return tuple(t.clone() for t in self.replay(*args))

    def release(self):
        """Drops the captured graph and its static buffers."""
        self._step.release()
