"""CPU oracle for the routed-MoE expert FFN path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this package.  The product (the CUDA library under
gfx906-qwen3.8fn_b200/) never loads it.

Two layers:
* `lib()` -- ctypes over oracle/liboracle.so, the plain-C restatement in
  oracle/moe_oracle.c (built by `build()` with gcc -ffp-contract=off);
* `ref()` / `ref_native()` -- ctypes over oracle/_ref/libqwen_ref*.so, the
  reference's own CPU code built by oracle/build_ref.py (absent when the
  reference tree was not available at build time).

The numpy helpers below compose the restated functions into a whole MoE layer
exactly as the reference's Layer::ffn does (src/session.hip:1412-1556):
quantise x, softmax, select_routes, group, per-(token, rank) expert, rank-order
fold, shared expert with sigmoid gate.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "moe_oracle.c")
SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqwen_ref.so")
REF_NATIVE_SO = os.path.join(HERE, "_ref", "libqwen_ref_native.so")

Q8_DTYPE = np.dtype([("d", "<u2"), ("s", "<u2"), ("qs", "i1", (32,))])
assert Q8_DTYPE.itemsize == 36
ASSIGN_DTYPE = np.dtype([("token", "<i4"), ("rank", "<i4"), ("expert", "<i4"), ("weight", "<f4")])

HIDDEN, INTER, EXPERTS, TOP_K = 2048, 512, 512, 10
Q4_BLOCK = 18
Q4_1_BLOCK = 20
Q4_0, Q4_1 = 2, 3          # TensorType values of the reference (src/model.hpp:17-19)


def build(force=False):
    """Compile moe_oracle.c into liboracle.so (gcc, strict IEEE)."""
    if not force and os.path.exists(SO) and os.path.getmtime(SO) >= os.path.getmtime(SRC):
        return SO
    cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-fvisibility=hidden", SRC, "-o", SO, "-lm"]
    subprocess.run(cmd, check=True)
    return SO


_lib = None
_ref = {}

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
F = ctypes.c_float
U16 = ctypes.c_uint16
U32 = ctypes.c_uint32
U64 = ctypes.c_uint64


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(SO)
        sig = {
            "o_half_to_float": (F, [U16]),
            "o_float_to_half": (U16, [F]),
            "o_quantize_block": (I, [P, P]),
            "o_quantize_q8_1": (I, [P, SZ, P]),
            "o_block_dot": (I, [P, P]),
            "o_block_dots": (None, [P, P, I, I, I, P]),
            "o_expf_mismatches": (ctypes.c_int64, [P, ctypes.c_uint32, ctypes.c_uint32, P]),
            "o_matrix_serial": (None, [P, P, I, I, I, P]),
            "o_matrix_mmvq": (None, [P, P, I, I, I, P]),
            "o_expert_whole": (I, [P, P, P, I, I, P, I, P, P, P]),
            "o_expert_whole_typed": (I, [P, P, P, I, I, I, P, I, P, P, P]),
            "o_block_dots_q4_1": (None, [P, P, I, I, I, P]),
            "o_matrix_serial_q4_1": (None, [P, P, I, I, I, P]),
            "o_matrix_mmvq_q4_1": (None, [P, P, I, I, I, P]),
            "o_synth_q4_1": (None, [U64, U32, U32, U32, SZ, P]),
            "o_route_exp": (F, [F]),
            "o_router_softmax": (I, [P, I, P]),
            "o_select_routes": (I, [P, I, P, P]),
            "o_route_groups": (None, [P, P, I, I, I, P, P, P, P, P, P]),
            "o_routed_fold": (None, [P, P, I, I, P]),
            "o_shared_add": (None, [P, P, P, I, I, P]),
            "o_synth_base": (U64, [U64, U32, U32, U32]),
            "o_synth_q4_0": (None, [U64, U32, U32, U32, SZ, P]),
            "o_fixture_xorshift_q4_0": (None, [U32, SZ, P]),
            "o_fixture_xorshift_q4_1": (None, [U32, SZ, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _load_ref(path):
    if path in _ref:
        return _ref[path]
    if not os.path.exists(path):
        _ref[path] = None
        return None
    L = ctypes.CDLL(path)
    sig = {
        "ref_last_message": (ctypes.c_char_p, []),
        "ref_shape_hidden": (I, []),
        "ref_shape_inter": (I, []),
        "ref_half_to_float": (F, [U16]),
        "ref_float_to_half": (U16, [F]),
        "ref_quantize_q8": (I, [P, SZ, P]),
        "ref_matmul": (I, [I, I, I, I, P, SZ, P, SZ, I, P, SZ]),
        "ref_dot": (F, [I, I, P, P]),
        "ref_routes_new": (P, [I, I]),
        "ref_routes_free": (None, [P]),
        "ref_routes_prepare": (I, [P, P, P, SZ, I]),
        "ref_routes_assignments": (SZ, [P, P, SZ]),
        "ref_routes_counts": (None, [P, P]),
        "ref_expert_new": (P, [P, P, P, SZ, SZ, I, I]),
        "ref_expert_new_typed": (P, [P, P, P, I, SZ, SZ, I, I]),
        "ref_expert_free": (None, [P]),
        "ref_run_cpu_expert": (I, [P, I, P, SZ, I, P, SZ]),
        "ref_allowed_physical_cpus": (I, [P, SZ, ctypes.POINTER(SZ)]),
        "ref_pool_new": (P, [SZ, I, P, SZ]),
        "ref_pool_free": (None, [P]),
        "ref_pool_submit": (I, [P, P, I, P, SZ, I, P, SZ, ctypes.POINTER(SZ)]),
        "ref_pool_drain": (I, [P]),
        "ref_pool_reset": (I, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _ref[path] = L
    return L


def ref():
    """The reference's CPU code, CpuExpert shape-patched to 2048/512 (or None)."""
    return _load_ref(REF_SO)


def ref_native():
    """The reference's CPU code at its own 2560/640 expert shape (or None)."""
    return _load_ref(REF_NATIVE_SO)


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


# --------------------------------------------------------------------------- #
# numpy-level helpers over the C restatement
# --------------------------------------------------------------------------- #
def quantize(x):
    """float32 [..., n] -> (Q8_1 structured array [..., n/32], flags)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32, dtype=Q8_DTYPE)
    flags = lib().o_quantize_q8_1(ptr(x), x.size, ptr(out))
    return out.reshape(x.shape[:-1] + (x.shape[-1] // 32,)), flags


def synth_q4_0(seed, layer, expert, matrix, rows, blocks):
    """Canonical Q4_0 bytes [rows*blocks*18] of one generated matrix."""
    out = np.empty(rows * blocks * Q4_BLOCK, dtype=np.uint8)
    lib().o_synth_q4_0(seed, layer, expert, matrix, rows * blocks, ptr(out))
    return out


def synth_q4_1(seed, layer, expert, matrix, rows, blocks):
    """Canonical Q4_1 bytes [rows*blocks*20] of one generated matrix."""
    out = np.empty(rows * blocks * Q4_1_BLOCK, dtype=np.uint8)
    lib().o_synth_q4_1(seed, layer, expert, matrix, rows * blocks, ptr(out))
    return out


def synth_expert(seed, layer, expert, hidden=HIDDEN, inter=INTER, down_type=Q4_0):
    """(gate, up, down) canonical bytes; gate/up [inter][hidden/32] Q4_0, down
    [hidden][inter/32] of down_type (Q4_0 or Q4_1)."""
    down = (synth_q4_1 if down_type == Q4_1 else synth_q4_0)(seed, layer, expert, 2, hidden, inter // 32)
    return (synth_q4_0(seed, layer, expert, 0, inter, hidden // 32),
            synth_q4_0(seed, layer, expert, 1, inter, hidden // 32),
            down)


def fixture_xorshift_q4_0(seed, rows, blocks):
    """The reference cpu_expert test's seeded Q4_0 matrix (tests/cpu_expert_test.cpp:227-246)."""
    out = np.empty(rows * blocks * Q4_BLOCK, dtype=np.uint8)
    lib().o_fixture_xorshift_q4_0(seed, rows * blocks, ptr(out))
    return out


def fixture_xorshift_q4_1(seed, rows, blocks):
    """Q4_1 version of the reference cpu_expert test matrix (tests/cpu_expert_test.cpp:219-241)."""
    out = np.empty(rows * blocks * Q4_1_BLOCK, dtype=np.uint8)
    lib().o_fixture_xorshift_q4_1(seed, rows * blocks, ptr(out))
    return out


def matrix_mmvq(w, xq, rows, blocks):
    xq = np.ascontiguousarray(xq)
    cols = xq.size // blocks
    out = np.empty(cols * rows, dtype=np.float32)
    lib().o_matrix_mmvq(ptr(w), ptr(xq), rows, blocks, cols, ptr(out))
    return out.reshape(cols, rows)


def matrix_serial(w, xq, rows, blocks):
    xq = np.ascontiguousarray(xq)
    cols = xq.size // blocks
    out = np.empty(cols * rows, dtype=np.float32)
    lib().o_matrix_serial(ptr(w), ptr(xq), rows, blocks, cols, ptr(out))
    return out.reshape(cols, rows)


def block_dots(w, xq, rows, blocks):
    xq = np.ascontiguousarray(xq)
    cols = xq.size // blocks
    out = np.empty(cols * rows * blocks, dtype=np.int32)
    lib().o_block_dots(ptr(w), ptr(xq), rows, blocks, cols, ptr(out))
    return out.reshape(cols, rows, blocks)


def _q4_1_call(fn, w, xq, rows, blocks, dtype):
    xq = np.ascontiguousarray(xq)
    cols = xq.size // blocks
    out = np.empty(cols * rows * (blocks if dtype == np.int32 else 1), dtype=dtype)
    getattr(lib(), fn)(ptr(w), ptr(xq), rows, blocks, cols, ptr(out))
    return out.reshape((cols, rows, blocks) if dtype == np.int32 else (cols, rows))


def block_dots_q4_1(w, xq, rows, blocks):
    return _q4_1_call("o_block_dots_q4_1", w, xq, rows, blocks, np.int32)


def matrix_serial_q4_1(w, xq, rows, blocks):
    return _q4_1_call("o_matrix_serial_q4_1", w, xq, rows, blocks, np.float32)


def matrix_mmvq_q4_1(w, xq, rows, blocks):
    return _q4_1_call("o_matrix_mmvq_q4_1", w, xq, rows, blocks, np.float32)


def expert_whole(gate, up, down, xq, hidden=HIDDEN, inter=INTER, down_type=Q4_0):
    """Unweighted expert output [columns][hidden] (reference CpuExpert 'whole' order)."""
    xq = np.ascontiguousarray(xq)
    cols = xq.size // (hidden // 32)
    out = np.empty(cols * hidden, dtype=np.float32)
    scratch = np.empty(cols * inter * 3, dtype=np.float32)
    mq = np.zeros(cols * inter // 32, dtype=Q8_DTYPE)
    flags = lib().o_expert_whole_typed(ptr(gate), ptr(up), ptr(down), down_type, hidden, inter, ptr(xq), cols,
                                       ptr(out), ptr(scratch), ptr(mq))
    return out.reshape(cols, hidden), flags


def router_softmax(logits):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T = logits.shape[0]
    probs = np.empty_like(logits)
    flags = lib().o_router_softmax(ptr(logits), T, ptr(probs))
    return probs, flags


def select_routes(probs):
    probs = np.ascontiguousarray(probs, dtype=np.float32)
    T = probs.shape[0]
    ids = np.empty((T, TOP_K), dtype=np.int32)
    w = np.empty((T, TOP_K), dtype=np.float32)
    if lib().o_select_routes(ptr(probs), T, ptr(ids), ptr(w)) != 0:
        raise ValueError("invalid route denominator")
    return ids, w


def route_groups(ids, weights, experts=EXPERTS):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    T, k = ids.shape
    n = T * k
    counts = np.empty(experts, np.int32)
    offsets = np.empty(experts + 1, np.int32)
    tok, rank, exp = (np.empty(n, np.int32) for _ in range(3))
    wt = np.empty(n, np.float32)
    lib().o_route_groups(ptr(ids), ptr(weights), T, k, experts, ptr(counts), ptr(offsets),
                         ptr(tok), ptr(rank), ptr(exp), ptr(wt))
    return dict(counts=counts, offsets=offsets, token=tok, rank=rank, expert=exp, weight=wt)


def moe_layer(x, logits, experts_fn, shared, gate_vec, tokens=None, down_type=Q4_0, threads=1):
    """Whole-layer oracle for the given tokens (default: all).

    experts_fn(e) -> (gate, up, down) canonical bytes; shared = (gate, up, down);
    down matrices of down_type (Q4_0 or Q4_1).  `threads` > 1 runs the experts
    (and column ranges of the shared expert) on a thread pool: the C calls
    release the GIL and every column's result is independent of the split.
    Returns (out [len(tokens)][H], ids, weights, flags).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, H = x.shape
    if tokens is None:
        tokens = np.arange(T)
    tokens = np.asarray(tokens)
    sub_x = np.ascontiguousarray(x[tokens])
    xq, flags = quantize(sub_x)
    probs, f2 = router_softmax(logits[tokens])
    flags |= f2
    ids, w = select_routes(probs)
    n = len(tokens)
    contrib = np.zeros((n, TOP_K, H), np.float32)

    def one(e):
        cols = np.argwhere(ids == e)
        g, u, d = experts_fn(int(e))
        y, f = expert_whole(g, u, d, np.ascontiguousarray(xq[cols[:, 0]]), H, down_type=down_type)
        return cols, y, f

    experts = [int(e) for e in np.unique(ids)]
    if threads > 1 and len(experts) > 1:
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(max_workers=threads) as pool:
            results = list(pool.map(one, experts))
    else:
        results = [one(e) for e in experts]
    for cols, y, f in results:
        flags |= f
        contrib[cols[:, 0], cols[:, 1]] = y
    out = np.empty((n, H), np.float32)
    lib().o_routed_fold(ptr(contrib), ptr(np.ascontiguousarray(w)), n, H, ptr(out))
    if threads > 1 and n >= 64:
        from concurrent.futures import ThreadPoolExecutor
        step = (n + threads - 1) // threads
        parts = [(c, min(n, c + step)) for c in range(0, n, step)]
        with ThreadPoolExecutor(max_workers=threads) as pool:
            res = list(pool.map(lambda r: expert_whole(shared[0], shared[1], shared[2],
                                                       np.ascontiguousarray(xq[r[0]:r[1]]), H,
                                                       down_type=down_type), parts))
        ys = np.concatenate([y for y, _ in res])
        for _, f in res:
            flags |= f
    else:
        ys, f = expert_whole(shared[0], shared[1], shared[2], xq, H, down_type=down_type)
        flags |= f
    gv = np.ascontiguousarray(gate_vec, dtype=np.float32)
    lib().o_shared_add(ptr(sub_x), ptr(gv), ptr(ys), n, H, ptr(out))
    return out, ids, w, flags
