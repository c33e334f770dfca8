"""Per-device counters that invalidate captured CUDA graphs.

Same contract as fast_moss/storage_epoch.py:1-18: `advance` bumps the
storage epoch (and, for a context change, the lifecycle counter); a graph
captured under an older epoch refuses to replay.
"""

_epochs = {}
_contexts = {}


def current(device):
    return _epochs.get(device, 0)


def advance(device, *, context=False):
    _epochs[device] = current(device) + 1
    if context:
        _contexts[device] = lifecycle(device) + 1


def lifecycle(device):
    return _contexts.get(device, 0)
