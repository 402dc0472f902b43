"""Typed errors of the device step: raised on the host when a kernel reports a failure.

The kernels never trap.  A bounded wait that expires (an mbarrier whose copy never landed, a peer
rank that never arrived at a cross-rank flag) writes a code into a device error word and returns;
the engine reads the words back with every decode step's tokens and raises ``DeviceStepError``
instead of emitting tokens computed from missing data.  Reference behaviour: DistComm's status-
tagged responses that unblock every rank with an error (internal/model/dist_collective.go:59-62).
"""
from __future__ import annotations


class DeviceStepError(RuntimeError):
    """A decode step's device error words were non-zero.

    kernel_code: the step's kernel word (1 = a bounded wait expired, 2 = an index out of range,
    3 = a bad argument, 4 = a peer rank never arrived at a fused GEMV all-reduce tile);
    collective_code: the collective kernels' word (1 = a peer rank never arrived at a barrier)."""

    def __init__(self, msg: str, kernel_code: int = 0, collective_code: int = 0):
        super().__init__(msg)
        self.kernel_code = kernel_code
        self.collective_code = collective_code
