"""CPU checks of the C ABI library: it builds, loads, exports every entry point that
include/*.h declares, and fails with a status (not an abort) where no GPU exists."""
import ctypes
import os
import re

import numpy as np

import lrs

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    inc = os.path.join(REPO, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            for m in re.finditer(r"\b(lrs_[a-z0-9_]+)\s*\(", src):
                names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(built_lib):
    L = ctypes.CDLL(built_lib)
    decl = declared_functions()
    assert len(decl) >= 13
    missing = [n for n in sorted(decl) if not hasattr(L, n)]
    assert not missing, missing
    assert decl <= set(lrs.EXPORTS) | decl
    assert set(lrs.EXPORTS) <= decl


def test_seed_state_is_seed_or_one(built_lib):
    L = lrs.lib()
    for s in (0, 1, 42, 0x1234_5678_9ABC_DEF0, 2**64 - 2):
        assert L.lrs_seed_state(s) == (s | 1)


def test_struct_layouts_match_header():
    assert lrs.PARAMS_DTYPE.itemsize == 24
    assert lrs.ROW_INFO_DTYPE.itemsize == 88


def test_create_without_gpu_returns_status(built_lib):
    import torch
    if torch.cuda.is_available():
        return
    L = lrs.lib()
    h = ctypes.c_void_p()
    rc = L.lrs_create(0, 4, 1000, 64, ctypes.byref(h))
    assert rc in (lrs.LRS_E_CUDA, lrs.LRS_E_INVALID)
    assert h.value is None
    assert L.lrs_last_error(None)


def test_invalid_arguments_are_rejected(built_lib):
    L = lrs.lib()
    h = ctypes.c_void_p()
    assert L.lrs_create(0, 0, 1000, 64, ctypes.byref(h)) == lrs.LRS_E_INVALID
    assert L.lrs_create(0, 4, 0, 64, ctypes.byref(h)) == lrs.LRS_E_INVALID
    assert L.lrs_create(0, 4, 1 << 23, 64, ctypes.byref(h)) == lrs.LRS_E_INVALID
    assert L.lrs_sample_device(None, None, 1, 1, 1, None, 0, None, None, None, None, None, None, None,
                               None) == lrs.LRS_E_INVALID
    st = ctypes.c_int(0)
    tok = L.lrs_sampler_sample(None, None, 0, None, None, 0, ctypes.byref(st))
    assert st.value == lrs.LRS_E_INVALID and tok == lrs.TOKEN_NONE
    assert L.lrs_poll_error(None) == lrs.LRS_E_INVALID
    assert L.lrs_noalloc_poll_error(-1, None) == lrs.LRS_E_INVALID
    assert L.lrs_noalloc_poll_error(0, None) == lrs.LRS_OK  # (no set-up yet on device 0: nothing to report)


def test_expf_table_matches_this_libm(built_lib):
    from lrs import build
    path = build.TABLE
    raw = open(path, "rb").read()
    assert raw[:8] == b"LRSEXPF1"
    count, lo, hi = np.frombuffer(raw[8:20], np.uint32)
    ent = np.frombuffer(raw[20:], np.uint32).reshape(-1, 2)
    assert len(ent) == count and count > 90_000
    assert (np.diff(ent[:, 0].astype(np.int64)) > 0).all()
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    xs = ent[::53, 0].view(np.float32)
    ys = ent[::53, 1].view(np.float32)
    got = np.array([libm.expf(float(x)) for x in xs], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), ys.view(np.uint32))
    # outside the table, correctly rounded exp equals libm's expf
    rng = np.random.default_rng(0)
    probe = -rng.random(20000).astype(np.float32) * 104
    table = set(ent[:, 0].tolist())
    for x in probe:
        if int(x.view(np.uint32)) in table:
            continue
        cr = np.float32(np.exp(np.float64(x)))
        assert np.float32(libm.expf(float(x))) == cr


def _midpoint_distance(x32):
    """Distance (float ulps) of exp(x) from the rounding midpoint next to it, as the
    loaders compute it (host double exp)."""
    d = np.exp(x32.astype(np.float64))
    c = d.astype(np.float32)
    up = d >= c.astype(np.float64)
    nb = np.where(up, np.nextafter(c, np.float32(np.inf)), np.nextafter(c, np.float32(0)))
    u = np.abs(nb.astype(np.float64) - c.astype(np.float64))
    return 0.5 - np.abs(d - c.astype(np.float64)) / u, c


def test_expf_entries_lie_near_midpoints():
    """The kernel answers an input without the table when its exp lies farther from a
    rounding midpoint than every table entry does; check that premise on this libm: the
    entries' largest distance is small, and sampled inputs farther than it have libm's
    value equal to the correctly rounded one."""
    from lrs import build
    raw = open(build.TABLE, "rb").read()
    ent = np.frombuffer(raw[20:], np.uint32).reshape(-1, 2)
    x = ent[:, 0].view(np.float32)
    dist, c = _midpoint_distance(x)
    normal = c >= np.float32(2.0 ** -126)
    near = max(float(dist[normal].max()), 2.0 ** -16) + 2.0 ** -20
    assert near < 2.0 ** -8  # (0.0016 ulp for glibc 2.39)
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    rng = np.random.default_rng(1)
    probe = (-rng.random(40000) * 104).astype(np.float32)
    pd, pc = _midpoint_distance(probe)
    normal_p = pc >= np.float32(2.0 ** -126)
    far = (pd > near) & normal_p
    assert far.sum() > 0.99 * normal_p.sum()  # (subnormal results always take the table)
    got = np.array([libm.expf(float(v)) for v in probe[far]], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), pc[far].view(np.uint32))
