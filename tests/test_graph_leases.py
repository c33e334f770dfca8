"""CPU: the resource leases that invalidate captured CUDA graphs
(fast_moss_b200.graphs).  An optimisation context opens a lease on its
device; a graph keeps the stamps of the leases open when it was captured
and may replay only while every one of them is still valid."""

import torch

from fast_moss_b200 import graphs


def test_lease_lifecycle_and_stamps():
    dev = torch.device("cuda", 7)  # a key only: no device is touched
    assert graphs.current_leases(dev) == ()
    a = graphs.open_lease(dev, owner="first")
    b = graphs.open_lease(dev, owner="second")  # two contexts may share a device
    assert graphs.current_leases(dev) == (a, b)
    stamps = (a.stamp(), b.stamp())
    assert graphs.CapturedStep._leases_valid((a, b), stamps)
    b.renew()  # the second context rebuilt a cached resource
    assert not graphs.CapturedStep._leases_valid((a, b), stamps)
    graphs.close_lease(b)
    assert graphs.current_leases(dev) == (a,)
    assert not b.valid(b.stamp())  # a revoked lease is never valid again
    s = a.stamp()
    graphs.close_lease(a)
    assert not a.valid(s)
    assert graphs.current_leases(dev) == ()
    assert graphs.current_leases(torch.device("cuda", 6)) == ()
