"""One-GPU tests of cail's multi-rank kernels with the ranks emulated.

The push two-shot and the one-shot allreduce of P ranks each run as one
cooperative launch on one GPU (libcail_kbench's cail_emulate_push and
cail_emulate_oneshot): every emulated rank has its own
input, output, workspace and flag array, and the ranks' CTAs synchronise
through the same release/acquire flags as across GPUs.  Oracle: the
rank-order fold acc = x_0; acc = op(acc, x_1); ... computed on the CPU with
torch (numpy for the unsigned types torch has no arithmetic for); the
kernel folds in the same order, so every result must match bit for bit.

Also: the copy and TMA bulk-copy kernels of the one-rank path, checked
against their source by the harness.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import LIB, gpu_count

pytestmark = pytest.mark.gpu

# storage classes (cail_elem_class_t order) -> numpy dtype
EC = [np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64, np.float32, np.float64]
OPS = ["sum", "prod", "max", "min"]


def _lib():
    if gpu_count() < 1:
        pytest.skip("needs a GPU")
    ctypes.CDLL(os.path.join(LIB, "libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    ctypes.CDLL(os.path.join(LIB, "libcail.so"), mode=ctypes.RTLD_GLOBAL)
    k = ctypes.CDLL(os.path.join(LIB, "libcail_kbench.so"))
    vp = ctypes.c_void_p
    for fn in (k.cail_emulate_push, k.cail_emulate_oneshot):
        fn.argtypes = [ctypes.c_int, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.c_size_t,
                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
    k.cail_bench_kernel_local.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_float)]
    return k


def _inputs(rng, dt, op, P, n):
    out = []
    for _ in range(P):
        if np.issubdtype(dt, np.floating):
            x = rng.uniform(0.999, 1.001, n) if op == "prod" else rng.standard_normal(n)
        elif op == "prod":
            x = rng.choice([1, -1], n) if np.issubdtype(dt, np.signedinteger) else rng.integers(1, 3, n)
        elif np.issubdtype(dt, np.signedinteger):
            x = rng.integers(-8, 9, n)
        else:
            x = rng.integers(0, 17, n)
        out.append(np.asarray(x).astype(dt))
    return out


def _fold(xs, op):
    """Rank-order fold on the CPU (torch where it has the dtype, else numpy;
    integers wrap, floats are IEEE in the element type)."""
    import torch

    dt = xs[0].dtype
    if dt in (np.uint16, np.uint32, np.uint64):
        acc = xs[0].copy()
        with np.errstate(over="ignore"):
            for x in xs[1:]:
                acc = {"sum": acc + x, "prod": acc * x, "max": np.where(acc > x, acc, x),
                       "min": np.where(acc < x, acc, x)}[op].astype(dt)
        return acc
    acc = torch.from_numpy(xs[0].copy())
    for x in xs[1:]:
        t = torch.from_numpy(x)
        acc = {"sum": lambda: acc + t, "prod": lambda: acc * t, "max": lambda: torch.where(acc > t, acc, t),
               "min": lambda: torch.where(acc < t, acc, t)}[op]()
    return acc.numpy()


def _signed_view(dt):
    return {np.uint16: np.int16, np.uint32: np.int32, np.uint64: np.int64}.get(dt, dt)


def _run(k, P, xs, op_i, ec, offset=0, in_place=False, G=0, piece=0, calls=2, options=1, expect_rc=0,
         kind="push"):
    """Uploads xs (one array per rank) at `offset` elements into fresh device
    buffers, runs the emulated kernel (kind: push or oneshot) and returns the
    P outputs."""
    import torch

    dt = xs[0].dtype
    n = xs[0].size
    sv = _signed_view(dt)
    srcs, dsts, keep = [], [], []
    for x in xs:
        buf = torch.empty(n + offset + 16, dtype=getattr(torch, np.dtype(sv).name), device="cuda")
        buf[offset:offset + n] = torch.from_numpy(x.view(sv)).cuda()
        s = buf[offset:offset + n]
        if in_place:
            d = s
        else:
            dbuf = torch.full((n + offset + 16,), 7, dtype=buf.dtype, device="cuda")
            d = dbuf[offset:offset + n]
            keep.append(dbuf)
        keep.append(buf)
        srcs.append(s)
        dsts.append(d)
    vp = ctypes.c_void_p
    sa = (vp * P)(*[s.data_ptr() for s in srcs])
    da = (vp * P)(*[d.data_ptr() for d in dsts])
    fn = k.cail_emulate_push if kind == "push" else k.cail_emulate_oneshot
    rc = fn(P, sa, da, n, ec, op_i, G, piece, 1 if in_place else calls, options)
    torch.cuda.synchronize()
    assert rc == expect_rc, f"cail_emulate_push returned {rc}"
    return [d.cpu().numpy().view(dt) for d in dsts]


KINDS = ["push", "oneshot"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("ec", range(10), ids=[np.dtype(t).name for t in EC])
@pytest.mark.parametrize("op", OPS)
def test_emulated_kernels_all_types_bit_exact(kind, ec, op):
    k = _lib()
    rng = np.random.default_rng(1000 + 10 * ec + OPS.index(op))
    for P, n in ((2, 4099), (3, 100003), (8, 1), (8, 7), (8, 65536 + 3)):
        xs = _inputs(rng, EC[ec], op, P, n)
        want = _fold(xs, op)
        for r, got in enumerate(_run(k, P, xs, OPS.index(op), ec, kind=kind)):
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (P, n, r)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("P", [2, 4, 5, 8])
def test_emulated_kernels_unaligned_and_in_place(kind, P):
    """Buffers one element off a 16-byte boundary take the element-wise path;
    in-place calls (input = output) must give the same result."""
    k = _lib()
    rng = np.random.default_rng(P)
    for ec, n in ((8, 300001), (1, 77777), (9, 4097)):
        xs = _inputs(rng, EC[ec], "sum", P, n)
        want = _fold(xs, "sum")
        for got in _run(k, P, xs, 0, ec, offset=1, kind=kind):
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (P, ec, n, "offset")
        for got in _run(k, P, xs, 0, ec, in_place=True, kind=kind):
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (P, ec, n, "in place")


@pytest.mark.parametrize("kind", KINDS)
def test_emulated_kernels_many_rounds(kind):
    """Few CTAs and small pieces: every CTA runs many rounds, so its slots
    rotate (two parities for the push two-shot, three slots for the
    one-shot) within one call and across calls."""
    k = _lib()
    rng = np.random.default_rng(5)
    for P, G, piece in ((2, 1, 256), (4, 3, 512), (8, 2, 1024)):
        xs = _inputs(rng, np.float32, "sum", P, 250007)
        want = _fold(xs, "sum")
        for got in _run(k, P, xs, 0, 8, G=G, piece=piece, calls=3, kind=kind):
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (kind, P, G, piece)


def test_device_checks_catch_an_inconsistent_argument():
    """CAIL_DEVICE_CHECKS: one round too few for the message (harmless
    unchecked: the end of the longest slice would stay unreduced) is caught
    before the kernel touches memory: status code 2, the outputs untouched
    (still 7), and the context usable for a correct call afterwards."""
    k = _lib()
    rng = np.random.default_rng(11)
    xs = _inputs(rng, np.float32, "sum", 4, 100000)
    outs = _run(k, 4, xs, 0, 8, G=2, piece=4096, calls=1, options=3, expect_rc=2)
    for got in outs:
        assert (got == 7).all()
    want = _fold(xs, "sum")
    for got in _run(k, 4, xs, 0, 8, G=2, piece=4096, calls=1, options=1):
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("kernel", [3, 5], ids=["bulk_copy", "copy"])
def test_one_rank_copy_kernels_copy_exactly(kernel):
    k = _lib()
    ms = ctypes.c_float(0)
    for nbytes in (16, 4096, (3 << 20) + 48, 256 << 20):
        assert k.cail_bench_kernel_local(kernel, 1, nbytes, 2, ctypes.byref(ms)) == 0, nbytes
