"""The failure path's host side (no GPU): after a failed piece, graph_compute
runs it again on the CUDA backend, as the reference runs it again on its
Vulkan sibling (src/ggml-zest.cpp:709-755,887-891). Here: the check that the
piece's inputs are intact (results go to their tensors as each op runs, and
ggml's allocator may place a result on an input it outlives), and the run
itself on the stand-in CUDA backend: host-memory inputs move into its memory
for the call (bytes intact, views at their offsets) and the tensors point
back afterwards; its failure is reported as a failure."""
import ctypes
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "ggml_harness"))
from harness import F32, I32, STATUS_FAILED, STATUS_SUCCESS, USAGE_COMPUTE, USAGE_WEIGHTS, Harness, Q8_0  # noqa: E402

_MEM = []  # host arrays the tensors point at, kept alive for the process


def mem(n_bytes: int, fill=None) -> int:
    a = np.zeros(n_bytes, dtype=np.uint8) if fill is None else np.asarray(fill).view(np.uint8).copy()
    _MEM.append(a)
    return a.ctypes.data


@pytest.fixture(scope="module")
def h():
    return Harness()


def test_inputs_intact_until_an_aliasing_result_is_written(h):
    # a = SCALE(x); b = ADD(a, x) placed on x's memory (the allocator's in-place reuse)
    dev = h.buffer(USAGE_COMPUTE)
    x_ptr = mem(64 * 8 * 4)
    x = h.tensor(F32, [64, 8], buffer=dev, data=x_ptr, name="x")
    a = h.scale(x, 2.0, buffer=dev, data=mem(64 * 8 * 4), name="a")
    b = h.add(a, x, buffer=dev, data=x_ptr, name="b")
    assert h.rerun_safe([a, b], failed_at=0), "only a was written: x is intact"
    assert not h.rerun_safe([a, b], failed_at=1), "b was written over x"
    assert not h.rerun_safe([a, b], failed_at=-1), "a failure at the end: everything may be written"


def test_no_alias_is_always_safe(h):
    dev = h.buffer(USAGE_COMPUTE)
    x = h.tensor(F32, [64, 8], buffer=dev, data=mem(64 * 8 * 4), name="x")
    a = h.scale(x, 2.0, buffer=dev, data=mem(64 * 8 * 4), name="a")
    b = h.add(a, x, buffer=dev, data=mem(64 * 8 * 4), name="b")
    for at in (0, 1, -1):
        assert h.rerun_safe([a, b], failed_at=at)


def test_a_view_of_an_input_counts_as_the_input(h):
    # the piece reads a view (rows 4..7) of x; b is written over those rows
    dev = h.buffer(USAGE_COMPUTE)
    x_ptr = mem(64 * 8 * 4)
    x = h.tensor(F32, [64, 8], buffer=dev, data=x_ptr, name="x")
    xv = h.tensor(F32, [64, 4], buffer=dev, data=x_ptr + 64 * 4 * 4, op="VIEW", src=(x,), view_src=x, name="xv")
    a = h.scale(xv, 2.0, buffer=dev, data=mem(64 * 4 * 4), name="a")
    b = h.add(a, a, buffer=dev, data=x_ptr + 64 * 4 * 4, name="b")
    assert h.rerun_safe([xv, a, b], failed_at=0)
    assert not h.rerun_safe([xv, a, b], failed_at=1)
    # written over rows 0..3 only: no overlap with the view
    b2 = h.add(a, a, buffer=dev, data=x_ptr, name="b2")
    assert h.rerun_safe([xv, a, b2], failed_at=1)


def test_a_view_of_a_result_is_not_an_input(h):
    # c reads a view of a (made in the piece): writing a is no reason to refuse
    dev = h.buffer(USAGE_COMPUTE)
    x = h.tensor(F32, [64, 8], buffer=dev, data=mem(64 * 8 * 4), name="x")
    a_ptr = mem(64 * 8 * 4)
    a = h.scale(x, 2.0, buffer=dev, data=a_ptr, name="a")
    av = h.tensor(F32, [64 * 8], buffer=dev, data=a_ptr, op="RESHAPE", src=(a,), view_src=a, name="av")
    c = h.scale(av, 3.0, buffer=dev, data=mem(64 * 8 * 4), name="c")
    assert h.rerun_safe([a, av, c], failed_at=-1)


def test_rerun_moves_host_inputs_and_points_back(h):
    h.sibling(status=STATUS_SUCCESS)
    dev = h.buffer(USAGE_COMPUTE)
    host = h.buffer(USAGE_COMPUTE, host=True)
    w = h.tensor(Q8_0, [256, 64], buffer=h.buffer(USAGE_WEIGHTS), data=mem(64 * 8 * 34), name="w")
    x = h.tensor(F32, [256, 32], buffer=dev, data=mem(256 * 32 * 4), name="x")
    mm = h.mul_mat(w, x, buffer=dev, data=mem(64 * 32 * 4), name="mm")
    positions = np.arange(32, dtype=np.int32) * 7 + 3
    pos_ptr = mem(0, positions)
    pos = h.tensor(I32, [32], buffer=host, data=pos_ptr, name="pos")
    q = h.rope(mm, pos, 64, 0, buffer=dev, data=mem(64 * 32 * 4), name="q")
    # a second host input reached only through a view (its last 16 values)
    table = np.linspace(1, 2, 48, dtype=np.float32)
    t_ptr = mem(0, table)
    t = h.tensor(F32, [48], buffer=host, data=t_ptr, name="t")
    tv = h.tensor(F32, [16], buffer=host, data=t_ptr + 32 * 4, op="VIEW", src=(t,), view_src=t, name="tv")
    s = h.add(q, tv, buffer=dev, data=mem(64 * 32 * 4), name="s")
    nodes = [mm, q, s]
    assert h.rerun(nodes) == STATUS_SUCCESS
    st = h.sibling_stats()
    assert st["runs"] == 1 and st["nodes"] == 3
    assert st["moved"] == 2, "the positions and the view of the table, in the CUDA backend's memory"
    want = int(positions.view(np.uint8).sum()) + int(table[32:].view(np.uint8).sum())
    assert st["moved_sum"] == want, "the moved bytes are the host tensors' bytes, the view at its offset"
    assert st["buffers"] == 1 and st["sets"] == 2, "one buffer; the two owners copied in"
    assert st["started"] == 1 and st["stopped"] == 1 and st["buffers_freed"] == 1
    # the tensors point back at host memory
    assert pos.data == pos_ptr and ctypes.cast(pos.buffer, ctypes.c_void_p).value == host
    assert t.data == t_ptr and tv.data == t_ptr + 32 * 4
    assert ctypes.cast(tv.buffer, ctypes.c_void_p).value == host


def test_rerun_reports_the_cuda_backend_failing(h):
    dev = h.buffer(USAGE_COMPUTE)
    x = h.tensor(F32, [64, 8], buffer=dev, data=mem(64 * 8 * 4), name="x")
    a = h.scale(x, 2.0, buffer=dev, data=mem(64 * 8 * 4), name="a")
    h.sibling(status=STATUS_FAILED)
    assert h.rerun([a]) == STATUS_FAILED
    assert h.sibling_stats()["runs"] == 1
    h.sibling(init_fails=True)
    assert h.rerun([a]) == STATUS_FAILED
    assert h.sibling_stats()["runs"] == 0, "no CUDA backend: nothing ran"
    h.sibling()
