"""Host-side Python mirror of libqwen_moe_b200.so (B200 routed-MoE expert FFN).

The product is the C ABI in include/qwen_moe_b200.h, implemented by CUDA
kernels for sm_100a in csrc/.  This module binds it with ctypes and keeps the
reference's host API names and error behaviour:

* `RouteGroups`  -- src/routes.hpp:28-65 (ValueError where the reference throws
  std::invalid_argument);
* `GpuExpert`    -- src/gpu_expert.hpp:7-21 (check_quantization / linear / run);
* `MoeLayer`, `MoeWeights` -- the routed-MoE FFN of src/session.hip:1412-1556
  as one device call (`forward`), plus parity taps (`route`, `quantize_q8_1`,
  `q4_linear`).

Device memory, streams and process groups come from PyTorch; tensors are
passed by pointer.  There is no CPU fallback: importing this module without
the built library raises, and every call goes to the GPU.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen_moe_b200.so")

MOE_OK, MOE_INVALID_ARGUMENT, MOE_NOT_SUPPORTED, MOE_CUDA_ERROR = 0, 1, 2, 3
MOE_NUMERIC_ERROR, MOE_TIMEOUT, MOE_OUT_OF_MEMORY = 4, 6, 7
MOE_OUT_ACCUMULATE, MOE_OUT_OVERWRITE = 0, 1
MOE_Q4_0, MOE_Q4_1 = 2, 3      # the reference's TensorType values (src/model.hpp:17-19)
HIDDEN, INTER, EXPERTS, TOP_K = 2048, 512, 512, 10

EXPORTED = [
    "moe_status_string", "moe_abi_version", "moe_last_error_message",
    "moe_weights_create", "moe_weights_destroy", "moe_weights_upload_expert",
    "moe_weights_upload_shared_gate", "moe_weights_synthesize", "moe_weights_download_expert",
    "moe_weights_expert_bytes", "moe_layer_create", "moe_layer_destroy", "moe_forward", "moe_forward_profiled",
    "moe_route",
    "moe_layer_read_flags", "moe_quantize_q8_1", "moe_q4_linear", "moe_expert_create",
    "moe_expert_destroy", "moe_expert_check_quantization", "moe_expert_linear", "moe_expert_run",
    "moe_route_groups_create", "moe_route_groups_destroy", "moe_route_groups_prepare",
    "moe_route_groups_assignments", "moe_route_groups_counts", "moe_route_groups_message",
    "moe_route_noalloc", "moe_ep_weights_create", "moe_ep_create", "moe_ep_destroy", "moe_ep_ipc_handle",
    "moe_ep_open_peers", "moe_ep_forward", "moe_ep_read_flags",
    "moe_weights_create_typed", "moe_ep_weights_create_typed", "moe_q4_1_linear", "moe_expert_create_typed",
    "moe_forward_contributions", "moe_weights_upload_router", "moe_forward_hidden", "moe_router_logits",
    "moe_ep_forward_hidden", "moe_debug_block_dots", "moe_debug_expf",
]


class MoeError(RuntimeError):
    """A CUDA/NCCL failure reported by the library (reference: std::runtime_error)."""

    def __init__(self, status, message):
        super().__init__(f"{message} [{status}]")
        self.status = status


class desc_t(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("inter", ctypes.c_int), ("experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("has_shared", ctypes.c_int), ("device", ctypes.c_int),
                ("max_tokens", ctypes.c_int)]


_lib = None
P, I, SZ, U64, U32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint32
DESC_P = ctypes.POINTER(desc_t)


def library(path=LIB_PATH):
    """Load the CUDA library; raise if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with __graft_entry__.build() "
                          "(python gfx906-qwen3.8fn_b200/build.py)")
    L = ctypes.CDLL(path)
    sig = {
        "moe_status_string": (ctypes.c_char_p, [I]),
        "moe_abi_version": (I, []),
        "moe_last_error_message": (ctypes.c_char_p, []),
        "moe_weights_create": (I, [DESC_P, ctypes.POINTER(P)]),
        "moe_weights_destroy": (I, [P]),
        "moe_weights_upload_expert": (I, [P, I, P, P, P, P]),
        "moe_weights_upload_shared_gate": (I, [P, P, P]),
        "moe_weights_synthesize": (I, [P, U64, U32, P]),
        "moe_weights_download_expert": (I, [P, I, P, P, P, P]),
        "moe_weights_expert_bytes": (SZ, [DESC_P]),
        "moe_layer_create": (I, [DESC_P, ctypes.POINTER(P)]),
        "moe_layer_destroy": (I, [P]),
        "moe_forward": (I, [P, P, P, P, I, P, I, P]),
        "moe_forward_profiled": (I, [P, P, P, P, I, P, I, P, ctypes.POINTER(P)]),
        "moe_route": (I, [P, P, I, P, P, P, P, P, P, P]),
        "moe_route_noalloc": (I, [P, I, P, P, P, P, P, P, P]),
        "moe_layer_read_flags": (I, [P, ctypes.POINTER(I), I, P]),
        "moe_quantize_q8_1": (I, [P, I, I, P, P, P]),
        "moe_q4_linear": (I, [P, I, I, P, I, P, P, P]),
        "moe_expert_create": (I, [P, P, P, I, I, I, I, ctypes.POINTER(P)]),
        "moe_expert_destroy": (I, [P]),
        "moe_expert_check_quantization": (I, [P, P, SZ, P]),
        "moe_expert_linear": (I, [P, I, I, P, I, P]),
        "moe_expert_run": (I, [P, P, I, P, I, ctypes.POINTER(ctypes.c_double),
                               ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
        "moe_route_groups_create": (I, [I, I, ctypes.POINTER(P)]),
        "moe_route_groups_destroy": (I, [P]),
        "moe_route_groups_prepare": (I, [P, P, P, SZ, I]),
        "moe_route_groups_assignments": (SZ, [P, P, SZ]),
        "moe_route_groups_counts": (I, [P, P]),
        "moe_route_groups_message": (ctypes.c_char_p, []),
        "moe_ep_weights_create": (I, [DESC_P, I, I, ctypes.POINTER(P)]),
        "moe_ep_weights_create_typed": (I, [DESC_P, I, I, I, ctypes.POINTER(P)]),
        "moe_weights_create_typed": (I, [DESC_P, I, ctypes.POINTER(P)]),
        "moe_q4_1_linear": (I, [P, I, I, P, I, P, P, P]),
        "moe_forward_contributions": (I, [P, P, P, P, I, P, P, P, I, P]),
        "moe_weights_upload_router": (I, [P, P, P]),
        "moe_forward_hidden": (I, [P, P, P, I, P, I, P]),
        "moe_router_logits": (I, [P, P, I, P, P]),
        "moe_ep_forward_hidden": (I, [P, P, P, I, P, I, P]),
        "moe_expert_create_typed": (I, [P, P, P, I, I, I, I, I, ctypes.POINTER(P)]),
        "moe_ep_create": (I, [DESC_P, I, I, ctypes.POINTER(P)]),
        "moe_ep_destroy": (I, [P]),
        "moe_ep_ipc_handle": (I, [P, P]),
        "moe_ep_open_peers": (I, [P, P]),
        "moe_ep_forward": (I, [P, P, P, P, I, P, I, P]),
        "moe_ep_read_flags": (I, [P, ctypes.POINTER(I), I, P]),
        "moe_debug_block_dots": (I, [P, P, P, P, I, I, I, P, P, P, P, P, P, P]),
        "moe_debug_expf": (I, [ctypes.c_uint32, ctypes.c_uint32, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status, message_fn=None):
    if status == MOE_OK:
        return
    L = library()
    msg = (message_fn or L.moe_last_error_message)().decode(errors="replace")
    if status == MOE_INVALID_ARGUMENT:
        raise ValueError(msg)
    if status == MOE_NOT_SUPPORTED:
        raise NotImplementedError(msg)
    raise MoeError(status, f"{L.moe_status_string(status).decode()}: {msg}")


def _ptr(t):
    """Device/host address of a torch tensor or numpy array (None -> NULL)."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return ctypes.c_void_p(t.data_ptr())
    return ctypes.c_void_p(t.ctypes.data)


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def make_desc(hidden=HIDDEN, inter=INTER, experts=EXPERTS, top_k=TOP_K, has_shared=1, device=0, max_tokens=8):
    return desc_t(hidden, inter, experts, top_k, has_shared, device, max_tokens)


class _Owned:
    """Owner of one library handle, released exactly once by close() or by the
    garbage collector (also during interpreter shutdown, when module globals
    may already be gone: the destroy entry point is bound at creation)."""

    _destroy_name = ""
    handle = None

    def _own(self, h):
        self._destroy = getattr(library(), self._destroy_name)
        self.handle = h

    def close(self):
        h, self.handle = self.handle, None
        if h:
            self._destroy(h)

    __del__ = close


class MoeWeights(_Owned):
    """Device-resident Q4_0 experts of one layer (routed + shared)."""

    _destroy_name = "moe_weights_destroy"

    def __init__(self, desc, down_type=MOE_Q4_0):
        self.desc, self.down_type = desc, down_type
        h = P()
        check(library().moe_weights_create_typed(ctypes.byref(desc), down_type, ctypes.byref(h)))
        self._own(h)

    def synthesize(self, seed, layer=0, stream=None):
        check(library().moe_weights_synthesize(self.handle, seed, layer, _stream(stream)))

    def upload_expert(self, expert, gate, up, down, stream=None):
        check(library().moe_weights_upload_expert(self.handle, expert, _ptr(gate), _ptr(up), _ptr(down),
                                                  _stream(stream)))

    def upload_shared_gate(self, gate_vec, stream=None):
        check(library().moe_weights_upload_shared_gate(self.handle, _ptr(gate_vec), _stream(stream)))

    def upload_router(self, router, stream=None):
        """ffn_gate_inp as host fp32 [512][H]."""
        import numpy as np
        router = np.ascontiguousarray(router, dtype=np.float32)
        if router.shape != (EXPERTS, self.desc.hidden):
            raise ValueError("router matrix must be fp32 [512][hidden]")
        check(library().moe_weights_upload_router(self.handle, _ptr(router), _stream(stream)))

    def router_logits(self, x, stream=None):
        """Router logits fp32 cuda [T][512] of x (cuda fp32 [T][H])."""
        import torch
        logits = torch.empty(x.shape[0], EXPERTS, device=x.device)
        check(library().moe_router_logits(self.handle, _ptr(x), x.shape[0], _ptr(logits), _stream(stream)))
        return logits

    def download_expert(self, expert, stream=None):
        import numpy as np
        d = self.desc
        blocks = d.hidden * d.inter // 32
        g, u = (np.empty(blocks * 18, np.uint8) for _ in range(2))
        w = np.empty(blocks * (20 if self.down_type == MOE_Q4_1 else 18), np.uint8)
        check(library().moe_weights_download_expert(self.handle, expert, _ptr(g), _ptr(u), _ptr(w),
                                                    _stream(stream)))
        return g, u, w



class MoeLayer(_Owned):
    """Workspace of one routed-MoE FFN layer; `forward` is the whole hot path."""

    _destroy_name = "moe_layer_destroy"

    def __init__(self, desc):
        self.desc = desc
        h = P()
        check(library().moe_layer_create(ctypes.byref(desc), ctypes.byref(h)))
        self._own(h)

    def forward(self, weights, x, logits, out, accumulate=True, stream=None):
        """out (+)= MoE(x).  x, out: fp32 cuda [T][H]; logits fp32 cuda [T][E]."""
        T = x.shape[0]
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        check(library().moe_forward(self.handle, weights.handle, _ptr(x), _ptr(logits), T, _ptr(out), flag,
                                    _stream(stream)))

    def forward_hidden(self, weights, x, out, accumulate=True, stream=None):
        """out (+)= MoE(x) with the router logits computed on the device."""
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        check(library().moe_forward_hidden(self.handle, weights.handle, _ptr(x), x.shape[0], _ptr(out), flag,
                                           _stream(stream)))

    def forward_contributions(self, weights, x, logits, out, accumulate=True, stream=None):
        """Deterministic trace mode: out (+)= the reference-order fold of the per-(token, rank)
        contributions.  Returns (contrib [T][10][H], shared [T][H] or None) as cuda tensors."""
        import torch
        T, H = x.shape
        contrib = torch.empty(T, TOP_K, H, device=x.device)
        shared = torch.empty(T, H, device=x.device) if self.desc.has_shared else None
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        check(library().moe_forward_contributions(self.handle, weights.handle, _ptr(x), _ptr(logits), T,
                                                  _ptr(contrib), _ptr(shared), _ptr(out), flag, _stream(stream)))
        return contrib, shared

    def forward_profiled(self, weights, x, logits, out, events, accumulate=True, stream=None):
        """forward() recording torch.cuda.Event objects [before gate/up, before down, after down]."""
        T = x.shape[0]
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        ev = (P * 3)(*[e.cuda_event for e in events])
        check(library().moe_forward_profiled(self.handle, weights.handle, _ptr(x), _ptr(logits), T, _ptr(out),
                                             flag, _stream(stream), ev))

    def route(self, logits, stream=None):
        """GPU routing tap: dict of cuda tensors probs/ids/weights/offsets/token/rank."""
        import torch
        T = logits.shape[0]
        dev = logits.device
        r = dict(probs=torch.empty(T, EXPERTS, device=dev), ids=torch.empty(T, TOP_K, dtype=torch.int32, device=dev),
                 weights=torch.empty(T, TOP_K, device=dev),
                 offsets=torch.empty(EXPERTS + 1, dtype=torch.int32, device=dev),
                 token=torch.empty(T * TOP_K, dtype=torch.int32, device=dev),
                 rank=torch.empty(T * TOP_K, dtype=torch.int32, device=dev))
        check(library().moe_route(self.handle, _ptr(logits), T, _ptr(r["probs"]), _ptr(r["ids"]),
                                  _ptr(r["weights"]), _ptr(r["offsets"]), _ptr(r["token"]), _ptr(r["rank"]),
                                  _stream(stream)))
        return r

    def block_dots(self, weights, x, logits, expert, max_pairs, stream=None):
        """Parity tap: forward (overwrite) recording expert `expert`'s per-block
        int32 dots.  Returns dict of cuda tensors gate/up [P][I][H/32], down
        [P][H][I/32], mid_codes [P][I], mid_ds [P][I/32] (half d | half s<<16)
        and out [T][H]."""
        import torch
        T, H = x.shape
        Ii = self.desc.inter
        dev = x.device
        r = dict(gate=torch.zeros(max_pairs, Ii, H // 32, dtype=torch.int32, device=dev),
                 up=torch.zeros(max_pairs, Ii, H // 32, dtype=torch.int32, device=dev),
                 down=torch.zeros(max_pairs, H, Ii // 32, dtype=torch.int32, device=dev),
                 mid_codes=torch.zeros(max_pairs, Ii, dtype=torch.int8, device=dev),
                 mid_ds=torch.zeros(max_pairs, Ii // 32, dtype=torch.int32, device=dev),
                 out=torch.empty(T, H, device=dev))
        check(library().moe_debug_block_dots(self.handle, weights.handle, _ptr(x), _ptr(logits), T, expert, max_pairs,
                                             _ptr(r["gate"]), _ptr(r["up"]), _ptr(r["down"]), _ptr(r["mid_codes"]),
                                             _ptr(r["mid_ds"]), _ptr(r["out"]), _stream(stream)))
        return r

    def read_flags(self, clear=True, stream=None):
        f = ctypes.c_int(0)
        check(library().moe_layer_read_flags(self.handle, ctypes.byref(f), int(clear), _stream(stream)))
        return f.value



EP_HANDLE_BYTES = 64


class EpWeights(MoeWeights):
    """Expert shard of rank `rank` of `world`: routed experts
    [rank*512/world, (rank+1)*512/world) as local 0.., then the shared expert."""

    def __init__(self, desc, rank, world, down_type=MOE_Q4_0):
        self.desc, self.down_type = desc, down_type
        self.rank, self.world = rank, world
        h = P()
        check(library().moe_ep_weights_create_typed(ctypes.byref(desc), rank, world, down_type, ctypes.byref(h)))
        self._own(h)


class EpLayer(_Owned):
    """One rank of the expert-parallel layer (one process per GPU).

    Peer buffers are mapped with CUDA IPC; `connect(exchange)` takes a
    function that all-gathers one bytes object per rank (for example
    `exchange_handles` over a torch.distributed group)."""

    _destroy_name = "moe_ep_destroy"

    def __init__(self, desc, rank, world):
        self.desc, self.rank, self.world = desc, rank, world
        h = P()
        check(library().moe_ep_create(ctypes.byref(desc), rank, world, ctypes.byref(h)))
        self._own(h)

    def ipc_handle(self):
        buf = ctypes.create_string_buffer(EP_HANDLE_BYTES)
        check(library().moe_ep_ipc_handle(self.handle, buf))
        return buf.raw

    def open_peers(self, handles):
        if len(handles) != self.world or any(len(b) != EP_HANDLE_BYTES for b in handles):
            raise ValueError("need one 64-byte handle per rank, in rank order")
        blob = ctypes.create_string_buffer(b"".join(handles), EP_HANDLE_BYTES * self.world)
        check(library().moe_ep_open_peers(self.handle, blob))

    def connect(self, exchange):
        self.open_peers(exchange(self.ipc_handle()))

    def forward(self, weights, x, logits, out, accumulate=True, stream=None):
        T = x.shape[0]
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        check(library().moe_ep_forward(self.handle, weights.handle, _ptr(x), _ptr(logits), T, _ptr(out), flag,
                                       _stream(stream)))

    def forward_hidden(self, weights, x, out, accumulate=True, stream=None):
        flag = MOE_OUT_ACCUMULATE if accumulate else MOE_OUT_OVERWRITE
        check(library().moe_ep_forward_hidden(self.handle, weights.handle, _ptr(x), x.shape[0], _ptr(out), flag,
                                              _stream(stream)))

    def read_flags(self, clear=True, stream=None):
        f = ctypes.c_int(0)
        check(library().moe_ep_read_flags(self.handle, ctypes.byref(f), int(clear), _stream(stream)))
        return f.value



def exchange_handles(handle, group=None):
    """All-gather one bytes object per rank over a torch.distributed group
    (any backend): the host-side plumbing of the peer mapping."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def route_noalloc(logits, error=None, stream=None):
    """moe_route_noalloc: routing with no device allocation by the library.

    For callers that cannot allocate device memory (work recorded under CUDA
    stream capture, hosts whose memory belongs to another allocator).  Outputs
    are the caller's tensors; the library's scratch is a static device array
    limited to 1024 tokens.  Returns dict ids/weights/offsets/token/rank and
    the error tensor."""
    import torch
    # the C entry point cannot see the tensor: check what it relies on
    if logits.dim() != 2 or logits.shape[1] != EXPERTS:
        raise ValueError("logits must be [tokens][512]")
    if logits.dtype != torch.float32 or not logits.is_contiguous():
        raise ValueError("logits must be contiguous float32")
    if logits.device.type != "cuda" or logits.device.index != torch.cuda.current_device():
        raise ValueError("logits must be on the current CUDA device (the static scratch is per device)")
    T = logits.shape[0]
    dev = logits.device
    r = dict(ids=torch.empty(T, TOP_K, dtype=torch.int32, device=dev), weights=torch.empty(T, TOP_K, device=dev),
             offsets=torch.empty(EXPERTS + 1, dtype=torch.int32, device=dev),
             token=torch.empty(T * TOP_K, dtype=torch.int32, device=dev),
             rank=torch.empty(T * TOP_K, dtype=torch.int32, device=dev))
    if error is None:
        error = torch.zeros(1, dtype=torch.int32, device=dev)
    check(library().moe_route_noalloc(_ptr(logits), T, _ptr(r["ids"]), _ptr(r["weights"]), _ptr(r["offsets"]),
                                      _ptr(r["token"]), _ptr(r["rank"]), _ptr(error), _stream(stream)))
    return r, error


def quantize_q8_1(x, error=None, stream=None):
    """fp32 cuda [columns][width] -> uint8 cuda [columns][width/32*36] canonical Q8_1."""
    import torch
    cols, width = x.shape
    q = torch.empty(cols, width // 32 * 36, dtype=torch.uint8, device=x.device)
    own = error is None
    if own:
        error = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(library().moe_quantize_q8_1(_ptr(x), width, cols, _ptr(q), _ptr(error), _stream(stream)))
    return q, error


def q4_linear(w_q4_0, rows, k, xq, columns, with_dots=False, stream=None):
    """Canonical Q4_0 (cuda uint8) x canonical Q8_1 (cuda uint8) -> fp32 [columns][rows] (+ int32 dots)."""
    import torch
    out = torch.empty(columns, rows, device=xq.device)
    dots = torch.empty(columns, rows, k // 32, dtype=torch.int32, device=xq.device) if with_dots else None
    check(library().moe_q4_linear(_ptr(w_q4_0), rows, k, _ptr(xq), columns, _ptr(out), _ptr(dots), _stream(stream)))
    return (out, dots) if with_dots else out


def q4_1_linear(w_q4_1, rows, k, xq, columns, with_dots=False, stream=None):
    """Canonical Q4_1 (cuda uint8, 20-byte blocks) x canonical Q8_1 -> fp32 [columns][rows] (+ int32 dots)."""
    import torch
    out = torch.empty(columns, rows, device=xq.device)
    dots = torch.empty(columns, rows, k // 32, dtype=torch.int32, device=xq.device) if with_dots else None
    check(library().moe_q4_1_linear(_ptr(w_q4_1), rows, k, _ptr(xq), columns, _ptr(out), _ptr(dots),
                                    _stream(stream)))
    return (out, dots) if with_dots else out


class RouteGroups(_Owned):
    """Host route grouping with the reference's contract (src/routes.hpp:28-65)."""

    CHUNK1024, LAYERWISE16384 = 0, 1
    _destroy_name = "moe_route_groups_destroy"

    def __init__(self, token_capacity, bound=CHUNK1024):
        h = P()
        L = library()
        check(L.moe_route_groups_create(token_capacity, bound, ctypes.byref(h)), L.moe_route_groups_message)
        self._own(h)
        self.capacity = token_capacity

    def prepare(self, ids, weights, tokens):
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        weights = np.ascontiguousarray(weights, dtype=np.float32).ravel()
        if ids.size != weights.size:
            raise ValueError("routes: expected exactly tokens*10 IDs and weights")
        L = library()
        check(L.moe_route_groups_prepare(self.handle, _ptr(ids), _ptr(weights), ids.size, tokens),
              L.moe_route_groups_message)

    def assignments(self):
        import numpy as np
        L = library()
        n = L.moe_route_groups_assignments(self.handle, None, 0)
        out = np.empty(n, dtype=[("token", "<i4"), ("rank", "<i4"), ("expert", "<i4"), ("weight", "<f4")])
        L.moe_route_groups_assignments(self.handle, _ptr(out), n)
        return out

    def counts(self):
        import numpy as np
        c = np.empty(EXPERTS, np.int32)
        library().moe_route_groups_counts(self.handle, _ptr(c))
        return c

    def group(self, expert):
        if not 0 <= expert < EXPERTS:
            raise ValueError("routes: group expert must be 0..511")
        c = self.counts()
        a = self.assignments()
        start = int(c[:expert].sum())
        return a[start:start + int(c[expert])]



class GpuExpert(_Owned):
    """Single resident expert (src/gpu_expert.hpp:7-21) on the sm_100a kernels."""

    _destroy_name = "moe_expert_destroy"

    def __init__(self, gate, up, down, device=0, max_columns=8, hidden=HIDDEN, inter=INTER, down_type=MOE_Q4_0):
        h = P()
        check(library().moe_expert_create_typed(_ptr(gate), _ptr(up), _ptr(down), down_type, hidden, inter, device,
                                                max_columns, ctypes.byref(h)))
        self._own(h)
        self.hidden, self.inter = hidden, inter

    def check_quantization(self, x, expected_q8):
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        e = np.ascontiguousarray(expected_q8)
        st = library().moe_expert_check_quantization(self.handle, _ptr(x), x.size, _ptr(e))
        if st == MOE_NUMERIC_ERROR:
            raise RuntimeError("CPU/GPU Q8_1 ABI mismatch")
        check(st)

    def linear(self, down, up, q8, columns):
        import numpy as np
        rows = self.hidden if down else self.inter
        out = np.empty((columns, rows), np.float32)
        q8 = np.ascontiguousarray(q8)
        check(library().moe_expert_linear(self.handle, int(down), int(up), _ptr(q8), columns, _ptr(out)))
        return out

    def run(self, x, columns, repeats=1):
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((columns, self.hidden), np.float32)
        t = [ctypes.c_double() for _ in range(3)]
        check(library().moe_expert_run(self.handle, _ptr(x), columns, _ptr(out), repeats, *map(ctypes.byref, t)))
        return out, dict(upload_ms=t[0].value, resident_ms=t[1].value, completed_wall_ms=t[2].value)

