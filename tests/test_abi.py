"""CPU tests of the C-ABI library: it loads without a GPU, exports every
function include/*.h declares, and its host RouteGroups keeps the reference
contract (tests/routes_test.cpp semantics) -- no device calls here."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

from conftest import ROOT, golden


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names.update(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol(pkg):
    L = pkg.library()
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    assert set(names) <= set(pkg.EXPORTED) | set(names)
    assert L.moe_abi_version() >> 16 == 1


def test_status_strings(pkg):
    L = pkg.library()
    assert L.moe_status_string(0) == b"ok"
    assert L.moe_status_string(1) == b"invalid_argument"
    assert L.moe_status_string(6) == b"timeout"


def test_invalid_descriptions_rejected_before_any_device_call(pkg):
    L = pkg.library()
    h = ctypes.c_void_p()
    for bad in (dict(hidden=100), dict(inter=48), dict(experts=256), dict(top_k=8), dict(max_tokens=0),
                dict(has_shared=2)):
        d = pkg.make_desc(**bad)
        st = L.moe_layer_create(ctypes.byref(d), ctypes.byref(h))
        assert st in (pkg.MOE_INVALID_ARGUMENT, pkg.MOE_NOT_SUPPORTED)
        assert not h.value
    with pytest.raises(ValueError):
        pkg.MoeLayer(pkg.make_desc(hidden=2049))
    with pytest.raises(NotImplementedError):
        pkg.MoeWeights(pkg.make_desc(experts=128))


def test_route_groups_matches_reference_golden(pkg):
    g = golden("routes.npz")
    for key in [k[:-4] for k in g.files if k.endswith("_ids")]:
        ids, w = g[key + "_ids"], g[key + "_weights"]
        tokens = ids.size // 10
        rg = pkg.RouteGroups(128)
        rg.prepare(ids, w, tokens)
        a = rg.assignments()
        want = g[key + "_assign"]
        got = np.stack([a["token"], a["rank"], a["expert"], a["weight"].view(np.int32)], 1)
        assert np.array_equal(got, want), key
        assert np.array_equal(rg.counts(), g[key + "_counts"])
        for e in (0, 41, 511):
            grp = rg.group(e)
            assert np.all(grp["expert"] == e)


def test_route_groups_rejections_leave_views_unchanged(pkg):
    rg = pkg.RouteGroups(4)
    ids = np.array([[(7 * t + 3 * r) % 512 for r in range(10)] for t in range(4)], np.int32)
    w = np.full((4, 10), 0.25, np.float32)
    rg.prepare(ids, w, 4)
    before = rg.assignments().copy()
    bad_cases = []
    dup = ids.copy(); dup[1, 9] = dup[1, 0]; bad_cases.append((dup, w, 4))
    oob = ids.copy(); oob[0, 0] = 512; bad_cases.append((oob, w, 4))
    neg = ids.copy(); neg[2, 3] = -1; bad_cases.append((neg, w, 4))
    for v in (np.nan, np.inf, -1.0):
        ww = w.copy(); ww[3, 4] = v; bad_cases.append((ids, ww, 4))
    bad_cases.append((ids, w, 5))   # above capacity
    bad_cases.append((ids, w, 0))
    bad_cases.append((ids[:3], w[:3], 4))  # wrong extent
    for i, ww, t in bad_cases:
        with pytest.raises(ValueError):
            rg.prepare(i, ww, t)
        assert np.array_equal(rg.assignments(), before)
    # negative zero weights are valid and kept bit-exact
    w2 = w.copy(); w2[0, 0] = -0.0
    rg.prepare(ids, w2, 4)
    assert rg.assignments()["weight"].view(np.uint32).tolist().count(0x80000000) == 1


def test_route_groups_capacity_bounds(pkg):
    for cap in (0, -1, 1025):
        with pytest.raises(ValueError):
            pkg.RouteGroups(cap)
    pkg.RouteGroups(1024)
    pkg.RouteGroups(16384, pkg.RouteGroups.LAYERWISE16384)
    with pytest.raises(ValueError):
        pkg.RouteGroups(16385, pkg.RouteGroups.LAYERWISE16384)
    with pytest.raises(ValueError):
        pkg.RouteGroups(4).group(512)


def test_route_groups_all_experts_large_batch(pkg, O):
    rng = np.random.default_rng(4)
    T = 1024
    ids = np.stack([rng.permutation(512)[:10] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, 10)).astype(np.float32)
    rg = pkg.RouteGroups(T)
    rg.prepare(ids, w, T)
    r = O.route_groups(ids, w)
    a = rg.assignments()
    assert np.array_equal(a["token"], r["token"]) and np.array_equal(a["rank"], r["rank"])
    assert np.array_equal(rg.counts(), r["counts"])


def test_new_entry_points_reject_before_any_device_call(pkg):
    """Typed weights, the Q4_1 tap, trace mode, router and hidden-state entry
    points validate their arguments before touching a device."""
    L = pkg.library()
    h = ctypes.c_void_p()
    d = pkg.make_desc(max_tokens=8)
    for bad_type in (0, 1, 8, 99):   # only Q4_0 (2) and Q4_1 (3) down matrices
        assert L.moe_weights_create_typed(ctypes.byref(d), bad_type, ctypes.byref(h)) == pkg.MOE_NOT_SUPPORTED
        assert L.moe_ep_weights_create_typed(ctypes.byref(d), 0, 1, bad_type, ctypes.byref(h)) == pkg.MOE_NOT_SUPPORTED
        assert not h.value
    assert L.moe_expert_create_typed(None, None, None, 9, 2048, 512, 0, 4, ctypes.byref(h)) in (
        pkg.MOE_INVALID_ARGUMENT, pkg.MOE_NOT_SUPPORTED)
    for rows, k, cols in ((0, 512, 1), (2048, 500, 1), (2048, 512, 0)):
        assert L.moe_q4_1_linear(None, rows, k, None, cols, None, None, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_q4_1_linear(None, 2048, 512, None, 1, None, None, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_forward_contributions(None, None, None, None, 8, None, None, None, 0, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_router_logits(None, None, 8, None, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_forward_hidden(None, None, None, 8, None, 0, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_ep_forward_hidden(None, None, None, 8, None, 0, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_weights_upload_router(None, None, None) == pkg.MOE_INVALID_ARGUMENT
    assert L.moe_abi_version() == (1 << 16) | 1
