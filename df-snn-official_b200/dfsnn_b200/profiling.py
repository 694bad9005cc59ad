"""Optional timing of the native calls (CUDA events on the launching stream).

Disabled by default (one global check per call).  When a NativeCallTimer is active, every
C-ABI call made by the autograd Functions is bracketed by a pair of CUDA events recorded
on the stream the kernels are launched on, together with the number of kernels the call
launches and its algorithmic HBM bytes (compulsory reads + writes), so a harness can
report per-kernel durations and achieved bandwidth measured inside its own timed region.
Calls made while the stream is being captured into a CUDA graph are counted only.

    with profiling.NativeCallTimer() as timer:
        ... run steps ...
    torch.cuda.synchronize()
    print(timer.summary())
"""
import contextlib
from collections import defaultdict

import torch

_ACTIVE = None


class NativeCallTimer:
    def __init__(self):
        self._events = defaultdict(list)     # name -> [(start, end)]
        self.launches = defaultdict(int)     # name -> kernels launched
        self.bytes = defaultdict(int)        # name -> algorithmic bytes moved
        self.calls = defaultdict(int)
        self._by_steps = defaultdict(list)   # (name, T) -> [(start, end, nbytes)]
        self.captured = defaultdict(int)     # name -> kernels recorded into a CUDA graph

    def __enter__(self):
        global _ACTIVE
        self._prev = _ACTIVE
        _ACTIVE = self
        return self

    def __exit__(self, *exc):
        global _ACTIVE
        _ACTIVE = self._prev
        return False

    def add(self, name, start, end, launches, nbytes, steps=None):
        self._events[name].append((start, end))
        self.launches[name] += launches
        self.bytes[name] += nbytes
        self.calls[name] += 1
        if steps is not None:
            self._by_steps[(name, steps)].append((start, end, nbytes))

    def summary_by_steps(self):
        """{f"{name}_T{T}": {calls, ms_per_call, bytes_per_call, gbs}} for the calls that gave
        their step count (call after synchronising the device)."""
        out = {}
        for (name, T), evs in sorted(self._by_steps.items()):
            ms = sum(s.elapsed_time(e) for s, e, _ in evs)
            nb = sum(b for _, _, b in evs)
            out[f"{name}_T{T}"] = {"calls": len(evs), "ms_per_call": ms / len(evs),
                                   "bytes_per_call": nb / len(evs),
                                   "gbs": (nb / 1e9) / (ms / 1e3) if ms > 0 else None}
        return out

    def summary(self):
        """{name: {calls, launches, ms_total, ms_per_call, bytes_per_call, gbs}} (call after
        synchronising the device)."""
        out = {}
        for name, evs in self._events.items():
            ms = sum(s.elapsed_time(e) for s, e in evs)
            calls = self.calls[name]
            out[name] = {
                "calls": calls,
                "launches": self.launches[name],
                "ms_total": ms,
                "ms_per_call": ms / calls,
                "bytes_per_call": self.bytes[name] / calls,
                "gbs": (self.bytes[name] / 1e9) / (ms / 1e3) if ms > 0 else None,
            }
        return out

    def total_launches(self):
        return sum(self.launches.values())

    def captured_launches(self):
        """Kernels recorded into CUDA graphs while the timer was active (each replay of such a
        graph launches them again)."""
        return sum(self.captured.values())


@contextlib.contextmanager
def native_call(name, launches, nbytes, device, steps=None):
    """Bracket one native call with CUDA events when a timer is active (`steps`: the call's T,
    for the per-T breakdown)."""
    timer = _ACTIVE
    if timer is None:
        yield
        return
    if torch.cuda.is_current_stream_capturing():
        # a capturing stream takes no timing events: count the kernels the graph will launch
        timer.captured[name] += launches
        yield
        return
    stream = torch.cuda.current_stream(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    yield
    end.record(stream)
    timer.add(name, start, end, launches, int(nbytes), steps)


# Algorithmic bytes per call (fp32 I/O): compulsory HBM reads + writes of one call.
def glmulti_forward_bytes(T, N, elem=4):
    return N * (2 * elem * T + 4)                # x in, spikes out (elem bytes each); v0 in


def glmulti_backward_bytes(T, N):
    return N * (12 * T + 8)                      # x, grad_spike in; grad_x out; v0 in, grad_v0 out


def schedule_forward_bytes(J, T):
    # masses, basis [J, T+1] and step powers in; scale [T], W [T, T] and c~ [T+1] out
    return 4 * (J + J * (T + 1) + J + T + T * T + T + 1)


def schedule_backward_bytes(J, T):
    # the forward's inputs and c~ in, grad_scale [T] and grad_W [T, T] in; grad masses [J] out
    return 4 * (J + J * (T + 1) + J + (T + 1) + T + T * T + J)


def single_forward_bytes(T, N):
    return N * (12 * T + 4 + 4 * ((T + 31) // 32))   # x in; spike, v, bits out; v0 in


def single_backward_bytes(T, N):
    return N * (16 * T + 4 + 4 * ((T + 31) // 32))   # grad_s, grad_v, v, bits in; grad_x, grad_v0 out


def single1_backward_bytes(T, N):
    return N * (16 * T + 8)                      # grad_s, grad_v, x in; grad_x out; v0 in, grad_v0 out


def history_forward_bytes(T, N, seqs_out):
    return N * (4 * T * (1 + seqs_out) + 4)      # x in; spike, v_pre, history (+ drift) out; v0 in


def history_backward_bytes(T, N, param_seqs):
    # compulsory: grad_spike, v_pre in; grad_x out; grad_v0 out; the saved sequences the
    # parameter gradients pair with grad_pre (param_seqs of them, 0 without parameter grads).
    # grad_pre itself is an intermediate (T = 8 and 16 never store it; other T write it and
    # read it back, 8 more bytes per neuron-step than counted here)
    return N * (4 * T * (3 + param_seqs) + 4)


def euler_forward_bytes(T, N):
    return N * (8 * T + 8)                       # x in, spikes out; z0 in, z_final out


def euler_backward_bytes(T, N):
    return N * (12 * T + 12)                     # x, grad_s in, grad_x out; z0, grad_zf in, grad_z0 out
