"""The phase-trace tool (kernelfoundry_b200.phase_trace) and the kernel's trace points agree.

CPU only: the tool's phase names follow kf::PrefillTracePoint in prefill_sm100.cuh slot for
slot, every point the tool names is stamped somewhere in the kernel, and the trace code is
compiled only under KF_PREFILL_TRACE (the shipped library exports no trace entry point)."""
import ctypes
import os
import re

from kernelfoundry_b200 import build, phase_trace

HEADER = os.path.join(build.CSRC, "prefill_sm100.cuh")


def _enum_names():
    src = open(HEADER).read()
    body = re.search(r"enum PrefillTracePoint \{(.*?)\};", src, re.S).group(1)
    return [n.strip().split("=")[0].strip() for n in body.replace("\n", " ").split(",") if n.strip()]


def test_phase_names_follow_the_enum():
    names = _enum_names()
    assert names[-1] == "kTrSlots" and names[-2] == "kTrSmid"
    points = names[:-2]
    assert len(points) == len(phase_trace.PHASES)
    assert names.index("kTrSmid") == phase_trace.SMID
    assert phase_trace.SLOTS == 32 and len(names) - 1 <= phase_trace.SLOTS


def test_every_point_is_stamped():
    src = open(HEADER).read()
    for n in _enum_names()[:-2]:
        if n in ("kTrEntry",):
            assert "KF_TRACE(kTrEntry)" in src
            continue
        base = re.sub(r"[01]$", "0", n)
        assert re.search(r"KF_TRACE\(" + base, src), n


def test_shipped_library_has_no_trace_entry_points():
    path = build.build()
    lib = ctypes.CDLL(path)
    for sym in ("kf_prefill_trace_read", "kf_prefill_trace_clear"):
        assert not hasattr(lib, sym), sym
