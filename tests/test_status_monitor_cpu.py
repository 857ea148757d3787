"""Host logic of the public API's kernel-status read-back (ops.flash.StatusMonitor):
a non-zero word reported by a finished call raises KernelStatusError at the next
poll, the word is re-armed, and calls that succeed raise nothing. The monitor
runs on a host tensor here (the read-back is a plain copy); the GPU tests drive
the same path with real kernels."""
import pytest
import torch


def test_error_word_raises_once_and_rearms():
    from multi_gpu_flashattention_b200.ops.flash import KernelStatusError, StatusMonitor
    m = StatusMonitor("cpu")
    m.after_launch("first call")
    m.poll()  # clean
    m.word.fill_(2 | (8 << 8) | (3 << 16))  # a kernel's peer-flag timeout at site 8, step 3
    m.after_launch("second call")
    m.after_launch("third call")  # the sticky word is read back again
    with pytest.raises(KernelStatusError, match=r"second call: peer flag wait timed out "
                                                r"\(code 2, site 8, step 3\)"):
        m.poll()
    assert int(m.word[0]) == 0 and not m.pending  # re-armed, later read-backs dropped
    m.after_launch("fourth call")
    m.poll(wait=True)


def test_depth_bounds_read_backs_in_flight():
    from multi_gpu_flashattention_b200.ops.flash import StatusMonitor
    m = StatusMonitor("cpu", depth=3)
    for i in range(10):
        m.after_launch(f"call {i}")
        assert len(m.pending) <= 3
    m.poll(wait=True)
    assert not m.pending and len(m._free) >= 1  # host slots are reused


def test_check_errors_covers_every_monitor():
    from multi_gpu_flashattention_b200.ops import flash
    m = flash.status_monitor("cpu")
    m.word.fill_(1)
    m.after_launch("host monitor")
    with pytest.raises(flash.KernelStatusError, match="mbarrier wait timed out"):
        flash.check_errors()
    flash.check_errors()  # re-armed
    flash._MONITORS.pop("cpu")
