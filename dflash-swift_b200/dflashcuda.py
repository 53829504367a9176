"""Python binding of libdflashcuda.so (ctypes over the C ABI in include/dflash_cuda.h).

Torch is used here only as device-memory and stream plumbing: tensors are handed to the
library as raw device pointers together with the current CUDA stream.  Every compute
call goes to the CUDA library; there is no CPU path.  If the shared library is missing
the import fails loudly.

Reference interface mirrored (random1st/dflash-swift):
  * ``SmallMQuantizedMatmul`` (Sources/DFlashKit/SmallMQuantizedMatmul.swift:27-225):
    ``apply``, ``is_eligible``, ``tiles``, row-count constants.
  * ``SmallMQuantizedLinear`` (:234-293): a quantized linear layer whose call routes
    through the kernel, sharing (never copying) the layer's packed arrays.
  * ``enable_small_m_quantized_matmul`` (:304-317): swaps every eligible layer of a
    module tree and returns how many were swapped (idempotent).
  * The gated-delta capture/replay used by rollbackGatedDeltaRound/Tree
    (DFlashSpeculativeGenerator.swift:450-461): ``gdn_step``, ``gdn_replay``,
    ``gdn_conv_rollback``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional, Sequence

HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DFLASH_CUDA_LIB", HERE / "libdflashcuda.so"))

DFLASH_OK = 0
DFLASH_ERR_INVALID_ARGUMENT = 1
DFLASH_ERR_UNSUPPORTED = 2
DFLASH_ERR_MISALIGNED = 3
DFLASH_ERR_CUDA = 4
DFLASH_ERR_NCCL = 5
DFLASH_ERR_TIMEOUT = 6
DFLASH_ERR_WORKSPACE = 7

DEVERR_QMM_PIPELINE = 0x1
DEVERR_QMM_REDUCE = 0x2
DEVERR_ALLREDUCE = 0x4
DEVERR_POSITION = 0x8
DEVERR_TEST_WAIT = 0x80000000

# Every symbol the header declares; tests check the library exports all of them.
EXPORTED = (
    "dflash_version", "dflash_last_error", "dflash_status_string", "dflash_device_error",
    "dflash_test_bounded_wait", "dflash_qmm_workspace_bytes", "dflash_qmm", "dflash_qmm_noalloc",
    "dflash_qmm_supported", "dflash_qmm_host_workspace_bytes", "dflash_qmm_host", "dflash_bias_add",
    "dflash_gdn_step", "dflash_gdn_replay", "dflash_gdn_conv_rollback",
    # include/dflash_stack.h: glue of the tensor-parallel verify stack
    "dflash_stack_add_rmsnorm", "dflash_stack_silu_mul", "dflash_stack_conv_silu", "dflash_stack_gdn_gates",
    "dflash_stack_gated_norm", "dflash_stack_attn_prep", "dflash_stack_attn_decode",
    "dflash_stack_add_rmsnorm_reduce", "dflash_tp_exchange_bytes", "dflash_tp_exchange_alloc",
    "dflash_tp_exchange_free", "dflash_ipc_get_handle", "dflash_ipc_open_handle", "dflash_ipc_close_handle",
    "dflash_tp_push", "dflash_qmm_ex", "dflash_accept", "dflash_stack_gdn_conv_gates",
    "dflash_accept_reduce",
    # speculative tree rounds
    "dflash_gdn_step_tree", "dflash_stack_gdn_conv_gates_tree", "dflash_stack_attn_prep_tree",
    "dflash_stack_attn_decode_tree", "dflash_stack_kv_compact", "dflash_accept_tree",
    # gated-delta layers with shared key heads
    "dflash_gdn_step_grouped", "dflash_gdn_step_tree_grouped", "dflash_gdn_replay_grouped",
    "dflash_stack_gdn_conv_gates_grouped",
    # attention with a device-resident cache position
    "dflash_stack_attn_prep_ex", "dflash_stack_attn_decode_ex",
    # the verify stack as one object
    "dflash_stack_create", "dflash_stack_forward", "dflash_stack_verify", "dflash_stack_commit",
    "dflash_stack_advance", "dflash_stack_context", "dflash_stack_output", "dflash_stack_destroy",
)


class DFlashError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_f = ctypes.c_float


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"libdflashcuda.so not found at {LIB_PATH}; build it with `python -c "
            f"'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "dflash_version": ([], _i),
        "dflash_last_error": ([], ctypes.c_char_p),
        "dflash_status_string": ([_i], ctypes.c_char_p),
        "dflash_device_error": ([ctypes.POINTER(ctypes.c_uint32), _vp], _i),
        "dflash_test_bounded_wait": ([ctypes.c_uint64, _vp], _i),
        "dflash_qmm_workspace_bytes": ([_i, _i, _i, _i, _i], _sz),
        "dflash_qmm": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp], _i),
        "dflash_qmm_noalloc": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp], _i),
        "dflash_qmm_supported": ([_i, _i, _i, _i], _i),
        "dflash_qmm_host_workspace_bytes": ([_i, _i, _i, _i, _i], _sz),
        "dflash_bias_add": ([_vp, _vp, _i, _i, _vp], _i),
        "dflash_qmm_host": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp], _i),
        "dflash_gdn_step": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, ctypes.c_float, _vp], _i),
        "dflash_gdn_replay": ([_vp, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(ctypes.c_int32), _i, _i, _i, _i,
                               _i, _i, _vp], _i),
        "dflash_gdn_conv_rollback": ([_vp, _vp, _vp, ctypes.POINTER(ctypes.c_int32), _i, _i, _i, _i, _i, _vp],
                                     _i),
        "dflash_stack_add_rmsnorm": ([_vp, _vp, _vp, _vp, _i, _i, _f, _vp], _i),
        "dflash_stack_silu_mul": ([_vp, _vp, _i, _i, _vp], _i),
        "dflash_stack_conv_silu": ([_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp], _i),
        "dflash_stack_gdn_gates": ([_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
        "dflash_stack_gated_norm": ([_vp, _vp, _i, _vp, _vp, _i, _i, _i, _f, _vp], _i),
        "dflash_stack_attn_prep": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _f, _vp], _i),
        "dflash_stack_attn_decode": ([_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp], _i),
        "dflash_stack_add_rmsnorm_reduce": ([_vp, _vp, _i, _i, _vp, _vp, _i, _i, _f, _vp], _i),
        "dflash_tp_exchange_bytes": ([_i, _i, _i], _sz),
        "dflash_tp_exchange_alloc": ([_sz, ctypes.POINTER(_vp)], _i),
        "dflash_tp_exchange_free": ([_vp], _i),
        "dflash_ipc_get_handle": ([_vp, _vp], _i),
        "dflash_ipc_open_handle": ([_vp, ctypes.POINTER(_vp)], _i),
        "dflash_ipc_close_handle": ([_vp], _i),
        "dflash_tp_push": ([_vp, ctypes.POINTER(_vp), _i, _i, _i, _i, _i, _vp], _i),
        "dflash_qmm_ex": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, ctypes.c_void_p, _vp], _i),
        "dflash_accept": ([_vp, _vp, _i, _vp, _vp, _vp], _i),
        "dflash_accept_reduce": ([_vp, _i, _i, _vp, _i, _vp, _vp, _vp], _i),
        "dflash_stack_gdn_conv_gates": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
                                        _i),
        "dflash_gdn_step_tree": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp], _i),
        "dflash_stack_gdn_conv_gates_tree": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i,
                                              _vp, _vp], _i),
        "dflash_stack_attn_prep_tree": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _f, _vp, _vp],
                                        _i),
        "dflash_stack_attn_decode_tree": ([_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp, _vp], _i),
        "dflash_stack_kv_compact": ([_vp, _vp, _i, ctypes.c_longlong, _i, _i, _i, _i,
                                     ctypes.POINTER(ctypes.c_int32), _i, _vp], _i),
        "dflash_accept_tree": ([_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp], _i),
        "dflash_gdn_step_grouped": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp], _i),
        "dflash_gdn_step_tree_grouped": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp], _i),
        "dflash_gdn_replay_grouped": ([_vp, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(ctypes.c_int32), _i, _i, _i, _i,
                                       _i, _i, _i, _vp], _i),
        "dflash_stack_gdn_conv_gates_grouped": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i,
                                                 _i, _vp, _vp], _i),
        "dflash_stack_attn_prep_ex": ([_vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _f, _vp, _vp, _vp],
                                      _i),
        "dflash_stack_attn_decode_ex": ([_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp], _i),
        "dflash_stack_create": ([_vp, _i, ctypes.POINTER(_vp)], _i),
        "dflash_stack_forward": ([_vp, _vp, _vp, _vp], _i),
        "dflash_stack_verify": ([_vp, _vp, _vp, _vp, _vp, _vp], _i),
        "dflash_stack_commit": ([_vp, ctypes.POINTER(ctypes.c_int32), _i, _vp], _i),
        "dflash_stack_advance": ([_vp, _i], _i),
        "dflash_stack_context": ([_vp], _i),
        "dflash_stack_output": ([_vp], _vp),
        "dflash_stack_destroy": ([_vp], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def last_error() -> str:
    return lib.dflash_last_error().decode()


def check(status: int) -> None:
    if status != DFLASH_OK:
        raise DFlashError(status, last_error())


def _stream(stream=None) -> int:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def device_error(stream=None) -> int:
    """Reads and clears the device error word (synchronises the stream)."""
    bits = ctypes.c_uint32(0)
    check(lib.dflash_device_error(ctypes.byref(bits), _stream(stream)))
    return int(bits.value)


def test_bounded_wait(limit_ns: int, stream=None) -> None:
    check(lib.dflash_test_bounded_wait(int(limit_ns), _stream(stream)))


# ----------------------------------------------------------------------------- qmm

def qmm_workspace_bytes(M: int, N: int, K: int, group_size: int, bits: int) -> int:
    return int(lib.dflash_qmm_workspace_bytes(M, N, K, group_size, bits))


class Workspace:
    """Zero-initialised device workspace for dflash_qmm (one per stream)."""

    def __init__(self, nbytes: int, device=None):
        import torch
        self.nbytes = int(nbytes)
        self.buf = torch.zeros(max(self.nbytes, 16), dtype=torch.uint8, device=device or "cuda")

    def ensure(self, nbytes: int) -> "Workspace":
        if nbytes > self.nbytes:
            self.__init__(nbytes, self.buf.device)
        return self


_workspaces: dict = {}


def default_workspace(nbytes: int, device) -> Workspace:
    import torch
    key = (str(device), torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None:
        ws = _workspaces[key] = Workspace(nbytes, device)
    return ws.ensure(nbytes)


def qmm(x, w, scales, biases, group_size: int, bits: int, out=None, workspace: Optional[Workspace] = None,
        stream=None):
    """y = x . dequant(w)^T through dflash_qmm.  x: bf16 [M, K] (M <= 16) on the GPU."""
    import torch
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    need = qmm_workspace_bytes(M, N, K, group_size, bits)
    ws = workspace.ensure(need) if workspace is not None else default_workspace(need, x.device)
    check(lib.dflash_qmm(_ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size, bits,
                         ws.buf.data_ptr(), ws.nbytes, _stream(stream)))
    return out


def qmm_host_workspace_bytes(M: int, N: int, K: int, group_size: int, bits: int) -> int:
    return int(lib.dflash_qmm_host_workspace_bytes(M, N, K, group_size, bits))


def qmm_host(x_host, w, scales, biases, group_size: int, bits: int, out_host=None,
             workspace: Optional[Workspace] = None, stream=None):
    """dflash_qmm_host: x bf16 [M, K] and the result in HOST memory (pinned for
    asynchronous copies), weights on the GPU; one library call queues copy in, matmul
    and copy out on the stream.  The result is valid after the stream has run past it."""
    import torch
    M, K = x_host.shape
    N = w.shape[0]
    if out_host is None:
        out_host = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    need = qmm_host_workspace_bytes(M, N, K, group_size, bits)
    ws = workspace.ensure(need) if workspace is not None else default_workspace(need, w.device)
    check(lib.dflash_qmm_host(_ptr(x_host), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out_host), M, N, K, group_size,
                              bits, ws.buf.data_ptr(), ws.nbytes, _stream(stream)))
    return out_host


def qmm_noalloc(x, w, scales, biases, group_size: int, bits: int, out=None, stream=None):
    """dflash_qmm without a workspace argument, for callers that may not allocate
    device memory: the library's own static device scratch is used instead (shapes up
    to its 8 MiB limit).  Calls on one device share the scratch: keep them ordered on
    one stream, or use qmm with one workspace per stream."""
    import torch
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    check(lib.dflash_qmm_noalloc(_ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size, bits,
                                 _stream(stream)))
    return out


class SmallMQuantizedMatmul:
    """Constants and dispatch of the small-M kernel (SmallMQuantizedMatmul.swift:27-225).

    The reference kernel only wins from 6 rows (below that MLX's GEMV is at roofline,
    :29-32) and stops at 16 (two 8-row MMA tiles, :36-37).  This library has no stock
    op to defer to, so its kernel covers every row count 1..16; wider inputs are cut
    into 16-row passes by SmallMQuantizedLinear.
    """

    minimum_rows = 1
    maximum_rows = 16
    rows_per_tile = 8
    supported_bits = (4, 8)
    supported_group_sizes = (32, 64, 128)

    @staticmethod
    def is_eligible(layer: "QuantizedLinear") -> bool:
        """Static half of the test (SmallMQuantizedMatmul.swift:193-201): affine mode
        with biases, a bit width and group size the kernel covers, and a shape it can
        tile."""
        if getattr(layer, "mode", "affine") != "affine" or layer.biases is None:
            return False
        out_features, in_features = layer.shape
        return bool(lib.dflash_qmm_supported(out_features, in_features, layer.group_size, layer.bits))

    @staticmethod
    def tiles(rows: int) -> int:
        """MMA n-tiles needed for `rows` (SmallMQuantizedMatmul.swift:205-207)."""
        return 1 if rows <= SmallMQuantizedMatmul.rows_per_tile else 2

    @staticmethod
    def apply(x, weight, scales, biases, rows: int, output_features: int, input_features: int, bits: int,
              group_size: int = 64):
        """x[rows, K] . deq(weight)^T -> [rows, N] bf16 (SmallMQuantizedMatmul.swift:210-224)."""
        assert x.shape[0] == rows and x.shape[1] == input_features and weight.shape[0] == output_features
        return qmm(x, weight, scales, biases, group_size, bits)


class QuantizedLinear:
    """MLX-layout affine-quantized linear layer: packed uint32 weight [N, K*bits/32],
    bf16 scales and biases [N, K/group_size], optional bf16 bias [N]."""

    def __init__(self, weight, scales, biases, group_size: int, bits: int, bias=None, mode: str = "affine"):
        self.weight, self.scales, self.biases, self.bias = weight, scales, biases, bias
        self.group_size, self.bits, self.mode = int(group_size), int(bits), mode
        self.frozen = False

    @property
    def shape(self):
        return (self.weight.shape[0], self.weight.shape[1] * 32 // self.bits)

    def freeze(self):
        self.frozen = True
        return self

    def __call__(self, x):
        raise NotImplementedError("the stock MLX quantizedMatmul is not part of this library; "
                                  "wrap the layer in SmallMQuantizedLinear")


class SmallMQuantizedLinear(QuantizedLinear):
    """QuantizedLinear whose forward runs on dflash_qmm (SmallMQuantizedMatmul.swift:234-293).

    Shares the wrapped layer's arrays (no copy) and stays frozen like the layer it
    replaces (:243-252).  The call flattens leading dimensions to rows (:255-256,
    :270), runs the kernel in passes of at most 16 rows (the kernel reads x rows in
    place, so the reference's zero-padding concat of :271-281 is not needed), reshapes
    back and adds the optional bias (:287-290).  Only bf16 input is accepted: the
    kernel's fragments and output are bf16 (:257-263); other dtypes raise TypeError
    rather than silently change the layer's output dtype.
    """

    def __init__(self, other: QuantizedLinear):
        super().__init__(other.weight, other.scales, other.biases, other.group_size, other.bits,
                         bias=other.bias, mode=other.mode)
        self.kernel_eligible = SmallMQuantizedMatmul.is_eligible(other)
        self.freeze()

    def __call__(self, x, stream=None):
        import torch
        if not self.kernel_eligible:
            raise DFlashError(DFLASH_ERR_UNSUPPORTED,
                              f"layer {self.shape} bits={self.bits} group={self.group_size} is not covered")
        if x.dtype != torch.bfloat16:
            raise TypeError(f"SmallMQuantizedLinear takes bfloat16 input, got {x.dtype}")
        lead = x.shape[:-1]
        K = x.shape[-1]
        N = self.weight.shape[0]
        flat = x.reshape(-1, K)
        if not flat.is_contiguous():
            flat = flat.contiguous()
        rows = flat.shape[0]
        y = torch.empty((rows, N), dtype=torch.bfloat16, device=x.device)
        step = SmallMQuantizedMatmul.maximum_rows
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            qmm(flat[r0:r1], self.weight, self.scales, self.biases, self.group_size, self.bits, out=y[r0:r1],
                stream=stream)
        if self.bias is not None and rows > 0:
            check(lib.dflash_bias_add(_ptr(y), _ptr(self.bias), rows, N, _stream(stream)))
        return y.reshape(*lead, N)


def enable_small_m_quantized_matmul(model) -> int:
    """Swaps every eligible QuantizedLinear in `model` for a SmallMQuantizedLinear
    (SmallMQuantizedMatmul.swift:304-317).  `model` is any object tree whose
    attributes (or list/dict items) hold layers.  Returns the number swapped; a second
    call returns 0 because wrapped layers are never wrapped again."""
    count = 0

    def visit(obj, seen):
        nonlocal count
        if id(obj) in seen:
            return
        seen.add(id(obj))
        items = []
        if isinstance(obj, dict):
            items = list(obj.items())
        elif isinstance(obj, (list, tuple)):
            items = list(enumerate(obj))
        elif hasattr(obj, "__dict__"):
            items = list(vars(obj).items())
        for key, child in items:
            if isinstance(child, QuantizedLinear):
                if isinstance(child, SmallMQuantizedLinear) or not SmallMQuantizedMatmul.is_eligible(child):
                    continue
                wrapped = SmallMQuantizedLinear(child)
                if isinstance(obj, dict):
                    obj[key] = wrapped
                elif isinstance(obj, list):
                    obj[key] = wrapped
                elif isinstance(obj, tuple):
                    continue
                else:
                    setattr(obj, key, wrapped)
                count += 1
            elif isinstance(child, (dict, list, tuple)) or (hasattr(child, "__dict__") and not _is_tensor(child)):
                visit(child, seen)

    visit(model, set())
    return count


def _is_tensor(obj) -> bool:
    return type(obj).__module__.startswith("torch")


# ----------------------------------------------------------------------------- gated delta

def gdn_step(state_in, state_out, q, k, v, alpha, beta, out=None, q_scale: float = 1.0, stream=None):
    """One layer's recurrence over T positions (the verify forward; its inputs are the capture).
    q, k [T, Hk, dk]; v [T, H, dv]: Hk < H shares each key head between H / Hk value heads."""
    T, Hk, dk = k.shape
    H, dv = v.shape[-2], v.shape[-1]
    args = (_ptr(state_in), _ptr(state_out), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(beta), _ptr(out), T, H)
    if Hk == H:
        check(lib.dflash_gdn_step(*args, dk, dv, float(q_scale), _stream(stream)))
    else:
        check(lib.dflash_gdn_step_grouped(*args, Hk, dk, dv, float(q_scale), _stream(stream)))
    return state_out


def gdn_step_tree(state_in, q, k, v, alpha, beta, parents, out, q_scale: float = 1.0, stream=None):
    """One layer's recurrence over the T rows of a tree round: row t gets the output of a
    chain over its root-to-t path from state_in.  parents: device int32 [T].  Key heads as
    for gdn_step."""
    T, Hk, dk = k.shape
    H, dv = v.shape[-2], v.shape[-1]
    args = (_ptr(state_in), _ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(beta), _ptr(parents), _ptr(out), T, H)
    if Hk == H:
        check(lib.dflash_gdn_step_tree(*args, dk, dv, float(q_scale), _stream(stream)))
    else:
        check(lib.dflash_gdn_step_tree_grouped(*args, Hk, dk, dv, float(q_scale), _stream(stream)))
    return out


def _rows_arg(rows: Optional[Sequence[int]]):
    if rows is None:
        return None
    arr = (ctypes.c_int32 * len(rows))(*[int(r) for r in rows])
    return arr


def gdn_replay(snapshot, state_out, k, v, alpha, beta, keep: int, rows: Optional[Sequence[int]] = None,
               stream=None):
    """Rollback replay for all layers at once.  k: [L, width, Hk, dk]; v: [L, width, H, dv];
    state: [L, H, dv, dk] (Hk < H: shared key heads, as for gdn_step)."""
    L, width, Hk, dk = k.shape
    H, dv = v.shape[-2], v.shape[-1]
    if rows is not None and len(rows) < keep:
        raise ValueError("rows shorter than keep")
    args = (_ptr(snapshot), _ptr(state_out), _ptr(k), _ptr(v), _ptr(alpha), _ptr(beta), _rows_arg(rows), int(keep),
            width, L, H)
    if Hk == H:
        check(lib.dflash_gdn_replay(*args, dk, dv, _stream(stream)))
    else:
        check(lib.dflash_gdn_replay_grouped(*args, Hk, dk, dv, _stream(stream)))
    return state_out


def gdn_conv_rollback(window, window_out, conv_in, keep: int, rows: Optional[Sequence[int]] = None, stream=None):
    """Conv-window rebuild.  window: [L, kc1, C]; conv_in: [L, width, C]."""
    L, kc1, C = window.shape
    width = conv_in.shape[1]
    if rows is not None and len(rows) < keep:
        raise ValueError("rows shorter than keep")
    check(lib.dflash_gdn_conv_rollback(_ptr(window), _ptr(window_out), _ptr(conv_in), _rows_arg(rows), int(keep),
                                       width, L, kc1, C, _stream(stream)))
    return window_out


# ----------------------------------------------------------------------------- verify-stack glue
# (include/dflash_stack.h; tensors row-major with one row per token)

def stack_add_rmsnorm(resid, delta, weight, out, eps: float, stream=None):
    M, H = resid.shape
    check(lib.dflash_stack_add_rmsnorm(_ptr(resid), _ptr(delta), _ptr(weight), _ptr(out), M, H, float(eps),
                                       _stream(stream)))
    return out


def stack_silu_mul(gate_up, out, stream=None):
    M, I = out.shape
    check(lib.dflash_stack_silu_mul(_ptr(gate_up), _ptr(out), M, I, _stream(stream)))
    return out


def stack_conv_silu(x, window, weight, out, channels: int, parts: int, stream=None):
    """x: [M, ld] (channels convolved at [0, channels)); window [kc-1, C]; out [parts, M, C/parts]."""
    M, ld = x.shape[0], x.stride(0)
    kc = weight.shape[1]
    check(lib.dflash_stack_conv_silu(_ptr(x), ld, _ptr(window), _ptr(weight), _ptr(out), M, channels, kc, parts,
                                     _stream(stream)))
    return out


def stack_gdn_gates(q, k, ab, a_log, dt_bias, alpha, beta, stream=None):
    """q, k: [M, H, dk] (normalised in place); ab: [M, ld] with b then a; alpha, beta [M, H] fp32."""
    M, H, dk = q.shape
    check(lib.dflash_stack_gdn_gates(_ptr(q), _ptr(k), _ptr(ab), ab.stride(0), _ptr(a_log), _ptr(dt_bias),
                                     _ptr(alpha), _ptr(beta), M, H, dk, _stream(stream)))


def stack_gated_norm(o, z, weight, out, eps: float, stream=None):
    """o: [M, H, dv]; z: [M, >= H*dv] rows; out: [M, H*dv]."""
    M, H, dv = o.shape
    check(lib.dflash_stack_gated_norm(_ptr(o), _ptr(z), z.stride(0), _ptr(weight), _ptr(out), M, H, dv, float(eps),
                                      _stream(stream)))
    return out


def stack_attn_prep(qkv, q_norm, k_norm, cache_k, cache_v, hq: int, hkv: int, rot: int, pos0: int, eps: float,
                    theta: float, stream=None, parents=None, position=None):
    """qkv rows [q | gate | k | v]; caches [hkv, max_len, d].  parents (device int32 [M]):
    a tree round, rotary position pos0 + depth.  position (device int32 [1]): pos0 read on
    the device instead (dflash_stack_attn_prep_ex)."""
    M = qkv.shape[0]
    _, max_len, d = cache_k.shape
    args = (_ptr(qkv), qkv.stride(0), _ptr(q_norm), _ptr(k_norm), _ptr(cache_k), _ptr(cache_v), M, hq, hkv, d, rot,
            pos0, max_len, float(eps), float(theta))
    if position is not None:
        check(lib.dflash_stack_attn_prep_ex(*args, _ptr(parents), _ptr(position), _stream(stream)))
    elif parents is None:
        check(lib.dflash_stack_attn_prep(*args, _stream(stream)))
    else:
        check(lib.dflash_stack_attn_prep_tree(*args, _ptr(parents), _stream(stream)))


def stack_attn_decode(qkv, cache_k, cache_v, out, hq: int, hkv: int, pos0: int, scale: float, stream=None,
                      parents=None, position=None):
    """parents (device int32 [M]): a tree round, each token sees the prefix and its path.
    position (device int32 [1]): pos0 read on the device (dflash_stack_attn_decode_ex)."""
    M = qkv.shape[0]
    _, max_len, d = cache_k.shape
    args = (_ptr(qkv), qkv.stride(0), _ptr(cache_k), _ptr(cache_v), _ptr(out), M, hq, hkv, d, pos0, max_len,
            float(scale))
    if position is not None:
        check(lib.dflash_stack_attn_decode_ex(*args, _ptr(parents), _ptr(position), _stream(stream)))
    elif parents is None:
        check(lib.dflash_stack_attn_decode(*args, _stream(stream)))
    else:
        check(lib.dflash_stack_attn_decode_tree(*args, _ptr(parents), _stream(stream)))
    return out


def accept_tree(target_tokens, parents, tokens, path, path_len, next_token, stream=None):
    """The accepted path of a tree round on the device: target_tokens, parents, tokens
    int32 [rows]; writes path int32 [rows] (first path_len entries), path_len [1],
    next_token [1]."""
    check(lib.dflash_accept_tree(_ptr(target_tokens), _ptr(parents), _ptr(tokens), tokens.shape[0], _ptr(path),
                                 _ptr(path_len), _ptr(next_token), _stream(stream)))


def stack_kv_compact(cache_k, cache_v, pos0: int, rows: Sequence[int], stream=None):
    """After a tree round: cache rows pos0 + rows[i] -> pos0 + i.  Caches [hkv, max_len, d]
    (one layer) or [layers, hkv, max_len, d] (contiguous)."""
    if cache_k.dim() == 3:
        layers, (hkv, max_len, d), stride = 1, cache_k.shape, 0
    else:
        layers, hkv, max_len, d = cache_k.shape
        stride = cache_k.stride(0)
    check(lib.dflash_stack_kv_compact(_ptr(cache_k), _ptr(cache_v), layers, stride, hkv, d, pos0, max_len,
                                      _rows_arg(rows), len(rows), _stream(stream)))


# ----------------------------------------------------------------------------- tensor-parallel exchange

IPC_HANDLE_BYTES = 64


class PeerExchange:
    """This rank's exchange buffer for the peer all-reduce (include/dflash_stack.h), mapped
    into every rank of the node.  `handles` come from ``handle()`` on every rank (the
    host exchanges them, e.g. with torch.distributed.all_gather_object)."""

    def __init__(self, world: int, M: int, H: int):
        self.world, self.M, self.H = world, M, H
        self.nbytes = int(lib.dflash_tp_exchange_bytes(world, M, H))
        if self.nbytes == 0:
            raise DFlashError(DFLASH_ERR_INVALID_ARGUMENT, f"exchange of world {world}, [{M}, {H}] not supported")
        ptr = ctypes.c_void_p()
        check(lib.dflash_tp_exchange_alloc(self.nbytes, ctypes.byref(ptr)))
        self.ptr = ptr.value
        self.bases = None
        self._opened = []

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib.dflash_ipc_get_handle(self.ptr, buf))
        return buf.raw

    def connect(self, rank: int, handles) -> None:
        bases = []
        for r, h in enumerate(handles):
            if r == rank:
                bases.append(self.ptr)
                continue
            p = ctypes.c_void_p()
            check(lib.dflash_ipc_open_handle(ctypes.create_string_buffer(bytes(h), IPC_HANDLE_BYTES), ctypes.byref(p)))
            self._opened.append(p.value)
            bases.append(p.value)
        self.rank = rank
        self.bases = (ctypes.c_void_p * len(bases))(*bases)

    def connect_local(self, rank: int, ptrs) -> None:
        """Use buffers of this process as the ranks' buffers (single-process tests)."""
        self.rank = rank
        self.bases = (ctypes.c_void_p * len(ptrs))(*ptrs)

    def push(self, part, set_: int, stream=None) -> None:
        M, H = part.shape
        check(lib.dflash_tp_push(_ptr(part), self.bases, self.rank, self.world, M, H, set_, _stream(stream)))

    def close(self) -> None:
        for p in self._opened:
            lib.dflash_ipc_close_handle(p)
        self._opened = []
        if self.ptr:
            lib.dflash_tp_exchange_free(self.ptr)
            self.ptr = None


def stack_add_rmsnorm_reduce(resid, exchange: PeerExchange, set_: int, weight, out, eps: float, stream=None):
    M, H = resid.shape
    check(lib.dflash_stack_add_rmsnorm_reduce(_ptr(resid), exchange.ptr, exchange.world, set_, _ptr(weight), _ptr(out),
                                              M, H, float(eps), _stream(stream)))
    return out


class QmmOptions(ctypes.Structure):
    """dflash_qmm_options (include/dflash_stack.h)."""
    _fields_ = [("x_swiglu", ctypes.c_int), ("push", ctypes.c_int), ("rank", ctypes.c_int), ("world", ctypes.c_int),
                ("set", ctypes.c_int), ("bases", ctypes.c_void_p), ("argmax_keys", ctypes.c_void_p),
                ("argmax_index_base", ctypes.c_int)]


def qmm_ex(x, w, scales, biases, group_size: int, bits: int, out=None, workspace: Optional[Workspace] = None,
           swiglu: bool = False, exchange: Optional[PeerExchange] = None, set_: int = 0, argmax_keys=None,
           argmax_index_base: int = 0, stream=None):
    """dflash_qmm_ex: with swiglu, x is [M, 2K] = [gate | up]; with an exchange, the result
    is pushed to every rank's exchange slot (set `set_`) instead of written to `out`; with
    argmax_keys (int64 [M] on the device) each row is reduced to its argmax key instead."""
    import torch
    M = x.shape[0]
    K = x.shape[1] // 2 if swiglu else x.shape[1]
    N = w.shape[0]
    if out is None and exchange is None and argmax_keys is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    o = QmmOptions(int(bool(swiglu)), 0, 0, 1, 0, None, _ptr(argmax_keys), int(argmax_index_base))
    if exchange is not None:
        o.push, o.rank, o.world, o.set = 1, exchange.rank, exchange.world, int(set_)
        o.bases = ctypes.cast(exchange.bases, ctypes.c_void_p)
    need = qmm_workspace_bytes(M, N, K, group_size, bits)
    ws = workspace.ensure(need) if workspace is not None else default_workspace(need, x.device)
    check(lib.dflash_qmm_ex(_ptr(x), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size, bits,
                            ws.buf.data_ptr(), ws.nbytes, ctypes.addressof(o), _stream(stream)))
    return out


def lm_head_argmax(x, w, scales, biases, group_size: int, bits: int, keys=None, workspace=None, index_base: int = 0,
                   stream=None):
    """Argmax keys of x . deq(W)^T per row without writing the logits (int64 [M]); with
    index_base, W is a vocabulary shard starting at that row."""
    import torch
    if keys is None:
        keys = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    qmm_ex(x, w, scales, biases, group_size, bits, workspace=workspace, argmax_keys=keys,
           argmax_index_base=index_base, stream=stream)
    return keys


def accept(keys, proposals, tokens=None, accepted=None, stream=None):
    """dflash_accept: (target tokens int32 [drafts + 1], accepted int32 [1]) on the device."""
    import torch
    drafts = proposals.shape[0]
    if tokens is None:
        tokens = torch.empty(drafts + 1, dtype=torch.int32, device=keys.device)
    if accepted is None:
        accepted = torch.empty(1, dtype=torch.int32, device=keys.device)
    check(lib.dflash_accept(_ptr(keys), _ptr(proposals), drafts, _ptr(tokens), _ptr(accepted), _stream(stream)))
    return tokens, accepted


def stack_gdn_conv_gates(x, window, weight, out, ab, a_log, dt_bias, alpha, beta, heads: int, dk: int, stream=None,
                         parents=None, k_heads: Optional[int] = None):
    """Conv + SiLU + q/k normalisation + gates in one kernel; out [3, M, heads, dk].
    parents (device int32 [M]): a tree round, each row convolved along its path.  k_heads
    < heads: q and k have k_heads heads (dflash_stack_gdn_conv_gates_grouped); out then
    holds [q: M x k_heads dk | k: M x k_heads dk | v: M x heads dk] contiguously."""
    M = x.shape[0]
    if k_heads is not None and k_heads != heads:
        check(lib.dflash_stack_gdn_conv_gates_grouped(
            _ptr(x), x.stride(0), _ptr(window), _ptr(weight), _ptr(out), _ptr(ab), ab.stride(0), _ptr(a_log),
            _ptr(dt_bias), _ptr(alpha), _ptr(beta), M, heads, k_heads, dk, weight.shape[1], _ptr(parents),
            _stream(stream)))
        return out
    args = (_ptr(x), x.stride(0), _ptr(window), _ptr(weight), _ptr(out), _ptr(ab), ab.stride(0), _ptr(a_log),
            _ptr(dt_bias), _ptr(alpha), _ptr(beta), M, heads, dk, weight.shape[1])
    if parents is None:
        check(lib.dflash_stack_gdn_conv_gates(*args, _stream(stream)))
    else:
        check(lib.dflash_stack_gdn_conv_gates_tree(*args, _ptr(parents), _stream(stream)))
    return out


def accept_reduce(exchange: PeerExchange, set_: int, proposals, tokens=None, accepted=None, stream=None):
    """dflash_accept_reduce over the ranks' keys pushed into `exchange` (laid out for [M, 4])."""
    import torch
    drafts = proposals.shape[0]
    dev = proposals.device
    if tokens is None:
        tokens = torch.empty(drafts + 1, dtype=torch.int32, device=dev)
    if accepted is None:
        accepted = torch.empty(1, dtype=torch.int32, device=dev)
    check(lib.dflash_accept_reduce(exchange.ptr, exchange.world, int(set_), _ptr(proposals), drafts, _ptr(tokens),
                                   _ptr(accepted), _stream(stream)))
    return tokens, accepted


# ----------------------------------------------------------------------------- the verify stack object

class QWeight(ctypes.Structure):
    """dflash_qweight (include/dflash_stack.h)."""
    _fields_ = [("w", _vp), ("scales", _vp), ("biases", _vp), ("N", _i), ("K", _i)]


class StackLayer(ctypes.Structure):
    """dflash_stack_layer."""
    _fields_ = [("attention", _i), ("ln", _vp), ("post_ln", _vp), ("in_proj", QWeight), ("out_proj", QWeight),
                ("conv", _vp), ("a_log", _vp), ("dt_bias", _vp), ("gdn_norm", _vp), ("snapshot", _vp),
                ("window", _vp), ("qkv", QWeight), ("o_proj", QWeight), ("q_norm", _vp), ("k_norm", _vp),
                ("cache_k", _vp), ("cache_v", _vp), ("gate_up", QWeight), ("down", QWeight)]


class StackDesc(ctypes.Structure):
    """dflash_stack_desc."""
    _fields_ = [("layers", _i), ("hidden", _i), ("block", _i), ("gdn_heads", _i), ("gdn_key_heads", _i),
                ("gdn_dk", _i), ("gdn_dv", _i), ("conv_kernel", _i), ("attn_heads", _i), ("kv_heads", _i),
                ("head_dim", _i), ("rotary_dim", _i), ("max_len", _i), ("rope_theta", _f), ("eps", _f),
                ("group", _i), ("bits", _i), ("rank", _i), ("world", _i), ("vocab0", _i),
                ("layer", ctypes.POINTER(StackLayer)), ("final_norm", _vp), ("lm_head", QWeight),
                ("exchange", _vp), ("key_exchange", _vp)]


def _qweight(q) -> QWeight:
    return QWeight(_ptr(q.w), _ptr(q.scales), _ptr(q.biases), q.N, q.K) if q is not None else QWeight()


class CStack:
    """dflash_stack: the verify stack driven by the library alone (include/dflash_stack.h),
    built over the shard weights and state of a verify_stack.VerifyStack-shaped shard (the
    dicts of build_rank_weights / build_rank_state) — the same buffers, referenced.  The
    exchanges (world > 1) are PeerExchange objects already connected to every rank."""

    def __init__(self, cfg, plan, weights: dict, state: dict, context: int, exchange=None, key_exchange=None):
        p, w = plan, weights
        layers = []
        for L, S in zip(w["layers"], state["layers"]):
            if L["kind"] == "gdn":
                layers.append(StackLayer(0, _ptr(L["ln"]), _ptr(L["post_ln"]), _qweight(L["in_proj"]),
                                         _qweight(L["out_proj"]), _ptr(L["conv"]), _ptr(L["a_log"]),
                                         _ptr(L["dt_bias"]), _ptr(L["gdn_norm"]), _ptr(S["snapshot"]),
                                         _ptr(S["window"]), QWeight(), QWeight(), None, None, None, None,
                                         _qweight(L["gate_up"]), _qweight(L["down"])))
            else:
                layers.append(StackLayer(1, _ptr(L["ln"]), _ptr(L["post_ln"]), QWeight(), QWeight(), None, None,
                                         None, None, None, None, _qweight(L["qkv"]), _qweight(L["o_proj"]),
                                         _ptr(L["q_norm"]), _ptr(L["k_norm"]), _ptr(S["cache_k"]),
                                         _ptr(S["cache_v"]), _qweight(L["gate_up"]), _qweight(L["down"])))
        self._layers = (StackLayer * len(layers))(*layers)
        self._keep = (weights, state, exchange, key_exchange)  # referenced, not copied: keep alive
        max_len = next((S["cache_k"].shape[1] for S in state["layers"] if "cache_k" in S), context + cfg.block)
        self.desc = StackDesc(
            cfg.layers, cfg.hidden, cfg.block, p.gdn_heads, p.gdn_key_heads or p.gdn_heads, cfg.gdn_dk, cfg.gdn_dv,
            cfg.conv_kernel, p.attn_heads, p.kv_heads, cfg.head_dim, cfg.rotary_dim, max_len, cfg.rope_theta,
            cfg.eps, cfg.group, cfg.bits, p.rank, p.world, p.vocab0, self._layers, _ptr(w["final_norm"]),
            _qweight(w["lm_head"]), ctypes.cast(exchange.bases, _vp) if exchange is not None else None,
            ctypes.cast(key_exchange.bases, _vp) if key_exchange is not None else None)
        h = _vp()
        check(lib.dflash_stack_create(ctypes.byref(self.desc), int(context), ctypes.byref(h)))
        self.handle = h

    def forward(self, hidden, out=None, stream=None):
        check(lib.dflash_stack_forward(self.handle, _ptr(hidden), _ptr(out), _stream(stream)))
        return out

    def output_ptr(self) -> int:
        return lib.dflash_stack_output(self.handle)

    def verify(self, hidden, proposals, tokens, accepted, stream=None):
        check(lib.dflash_stack_verify(self.handle, _ptr(hidden), _ptr(proposals), _ptr(tokens), _ptr(accepted),
                                      _stream(stream)))
        return tokens, accepted

    def commit(self, keep: int, stream=None):
        check(lib.dflash_stack_commit(self.handle, None, int(keep), _stream(stream)))

    def advance(self, n: int):
        check(lib.dflash_stack_advance(self.handle, int(n)))

    @property
    def context(self) -> int:
        return int(lib.dflash_stack_context(self.handle))

    def close(self):
        if self.handle:
            lib.dflash_stack_destroy(self.handle)
            self.handle = None
