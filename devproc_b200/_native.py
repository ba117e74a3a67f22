"""ctypes binding of ``libdevproc_b200.so`` (the C ABI in include/devproc_b200.h).

The structures below mirror the header field for field; ``tests`` compile the
header with gcc and compare every ``sizeof``.  Loading is lazy so that the IR,
DSL and compiler import on machines without the library, but every GPU entry
point goes through ``lib()``, which raises ``DevProcError`` when the library
is missing: there is no fallback implementation of any kernel.
"""

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdevproc_b200.so"


class DevProcError(RuntimeError):
    """A C-ABI call failed; the message carries the library's error text."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {message}")


DP_OK, DP_ERR_ARG, DP_ERR_SHAPE, DP_ERR_CUDA, DP_ERR_UNSUPPORTED, DP_ERR_PLAN, DP_ERR_STATE, DP_ERR_DEVICE = range(8)
STATUS_NAMES = {0: "DP_OK", 1: "DP_ERR_ARG", 2: "DP_ERR_SHAPE", 3: "DP_ERR_CUDA", 4: "DP_ERR_UNSUPPORTED",
                5: "DP_ERR_PLAN", 6: "DP_ERR_STATE", 7: "DP_ERR_DEVICE"}

# element types
DP_U8, DP_I8, DP_I16, DP_I32, DP_I64, DP_F16, DP_BF16, DP_F32, DP_F64, DP_BOOL = range(10)
DP_TF32 = 10  # GEMM operands: fp32 storage, TF32 tensor-core math
DTYPE_CODE = {"uint8": DP_U8, "int8": DP_I8, "int16": DP_I16, "int32": DP_I32, "int64": DP_I64,
              "float16": DP_F16, "bfloat16": DP_BF16, "float32": DP_F32, "float64": DP_F64, "bool": DP_BOOL}

DP_DEVERR_NONE, DP_DEVERR_INDEX, DP_DEVERR_TIMEOUT = 0, 1, 2
DP_LAYOUT_NHWC, DP_LAYOUT_NCHW = 0, 1
(DP_RED_SUM, DP_RED_MAX, DP_RED_MIN, DP_RED_MEAN, DP_RED_ARGMAX, DP_RED_SOFTMAX, DP_RED_RMSNORM,
 DP_RED_LAYERNORM) = range(8)
DP_B_NK, DP_B_KN = 0, 1
DP_EPI_BIAS, DP_EPI_RELU, DP_EPI_GELU_ERF, DP_EPI_GELU_TANH, DP_EPI_RESIDUAL, DP_EPI_SILU = 1, 2, 4, 8, 16, 32
DP_EPI_SOFTMAX = 64
DP_EPI_MUL = 128
DP_EPI_ARGMAX = 256
DP_EPI_TF32SPLIT = 512

DP_REGION_MAX_OPERANDS, DP_REGION_MAX_RANK, DP_REGION_MAX_INSTR = 8, 6, 64
DP_REGION_MAX_CONST, DP_REGION_MAX_REGS = 32, 8
OP = {"load": 1, "store": 2, "const": 3, "chansel": 4, "add": 10, "sub": 11, "mul": 12, "div": 13,
      "max": 14, "min": 15, "neg": 20, "abs": 21, "relu": 22, "sigmoid": 23, "tanh": 24, "exp": 25,
      "gelu_erf": 26, "gelu_tanh": 27, "silu": 28, "mov": 29, "tf32": 30}

DP_PLAN_MAGIC, DP_PLAN_VERSION = 0x32425044, 1
DP_NOALLOC_ARENA_BYTES = 64 << 20
DP_RECORD_MAX_OPERANDS, DP_RECORD_PARAM_BYTES = 8, 1280
DP_SLOT_BOUND, DP_SLOT_ARENA = 0, 1
DP_K_PREPROC, DP_K_ROWREDUCE, DP_K_GEMM, DP_K_REGION, DP_K_EMBEDDING, DP_K_COPY, DP_K_ATTENTION, DP_K_ROPE, \
    DP_K_SPLITK, DP_K_ARGMAX_KEYS, DP_K_GEMM_SK = range(1, 12)
KERNEL_NAMES = {1: "preproc", 2: "rowreduce", 3: "gemm", 4: "region", 5: "embedding", 6: "copy", 7: "attention",
                8: "rope", 9: "splitk", 10: "argmax_keys", 11: "gemm_sk"}


class PreprocParams(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("in_h", ctypes.c_int32), ("in_w", ctypes.c_int32),
                ("channels", ctypes.c_int32), ("out_h", ctypes.c_int32), ("out_w", ctypes.c_int32),
                ("in_dtype", ctypes.c_int32), ("in_layout", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("out_layout", ctypes.c_int32), ("normalize", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("mean", ctypes.c_float * 4), ("stdv", ctypes.c_float * 4)]


class RowReduceParams(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("has_weight", ctypes.c_int32), ("has_bias", ctypes.c_int32), ("out_split", ctypes.c_int32),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("in_row_stride", ctypes.c_int64),
                ("out_row_stride", ctypes.c_int64), ("eps", ctypes.c_float), ("weight_offset", ctypes.c_float)]


class GemmParams(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64), ("ldr", ctypes.c_int64),
                ("batch", ctypes.c_int64), ("stride_a", ctypes.c_int64), ("stride_b", ctypes.c_int64),
                ("stride_c", ctypes.c_int64), ("stride_r", ctypes.c_int64),
                ("a_dtype", ctypes.c_int32), ("b_dtype", ctypes.c_int32), ("c_dtype", ctypes.c_int32),
                ("r_dtype", ctypes.c_int32), ("b_layout", ctypes.c_int32), ("epilogue", ctypes.c_int32),
                ("bias_dtype", ctypes.c_int32), ("alpha", ctypes.c_float),
                ("batch2", ctypes.c_int64), ("stride_a2", ctypes.c_int64), ("stride_b2", ctypes.c_int64),
                ("stride_c2", ctypes.c_int64), ("stride_r2", ctypes.c_int64)]


class SplitKParams(ctypes.Structure):
    _fields_ = [("gemm", GemmParams), ("splits", ctypes.c_int64), ("slice_stride", ctypes.c_int64)]


class StreamKParams(ctypes.Structure):
    _fields_ = [("gemm", GemmParams), ("workspace_bytes", ctypes.c_int64)]


class ArgmaxKeysParams(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int64), ("mode", ctypes.c_int32), ("out_dtype", ctypes.c_int32)]


class RegionDesc(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("n_in", ctypes.c_int32), ("n_out", ctypes.c_int32),
                ("n_instr", ctypes.c_int32), ("shape", ctypes.c_int64 * DP_REGION_MAX_RANK),
                ("dtype", ctypes.c_int32 * DP_REGION_MAX_OPERANDS),
                ("stride", (ctypes.c_int64 * DP_REGION_MAX_RANK) * DP_REGION_MAX_OPERANDS),
                ("instr", ctypes.c_uint32 * DP_REGION_MAX_INSTR),
                ("consts", ctypes.c_float * DP_REGION_MAX_CONST),
                ("offset", ctypes.c_int64 * DP_REGION_MAX_OPERANDS)]


class EmbeddingParams(ctypes.Structure):
    _fields_ = [("n_ids", ctypes.c_int64), ("vocab", ctypes.c_int64), ("dim", ctypes.c_int64),
                ("id_dtype", ctypes.c_int32), ("w_dtype", ctypes.c_int32)]


class AttentionParams(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("heads_kv", ctypes.c_int64), ("group", ctypes.c_int64),
                ("L", ctypes.c_int64), ("S", ctypes.c_int64), ("D", ctypes.c_int64), ("Dv", ctypes.c_int64),
                ("q_sb", ctypes.c_int64), ("q_sh", ctypes.c_int64), ("q_sl", ctypes.c_int64),
                ("k_sb", ctypes.c_int64), ("k_sh", ctypes.c_int64), ("k_ss", ctypes.c_int64),
                ("v_sb", ctypes.c_int64), ("v_sh", ctypes.c_int64), ("v_ss", ctypes.c_int64),
                ("o_sb", ctypes.c_int64), ("o_sh", ctypes.c_int64), ("o_sl", ctypes.c_int64),
                ("scale", ctypes.c_float), ("dtype", ctypes.c_int32)]


class RopeParams(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("rows", ctypes.c_int64),
                ("dim", ctypes.c_int64),
                ("x_sb", ctypes.c_int64), ("x_sh", ctypes.c_int64), ("x_sr", ctypes.c_int64),
                ("o_sb", ctypes.c_int64), ("o_sh", ctypes.c_int64), ("o_sr", ctypes.c_int64),
                ("t_sb", ctypes.c_int64), ("t_sh", ctypes.c_int64), ("t_sr", ctypes.c_int64),
                ("half_table", ctypes.c_int32), ("x_dtype", ctypes.c_int32), ("t_dtype", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class PlanHeader(ctypes.Structure):
    _fields_ = [("magic", ctypes.c_uint32), ("version", ctypes.c_uint32), ("n_slots", ctypes.c_uint32),
                ("n_records", ctypes.c_uint32), ("arena_bytes", ctypes.c_uint64), ("reserved", ctypes.c_uint64)]


class PlanSlot(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("dtype", ctypes.c_uint32), ("offset", ctypes.c_uint64),
                ("bytes", ctypes.c_uint64)]


class PlanRecord(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_uint32), ("n_operands", ctypes.c_uint32),
                ("operand", ctypes.c_int32 * DP_RECORD_MAX_OPERANDS),
                ("params", ctypes.c_uint8 * DP_RECORD_PARAM_BYTES)]


PARAM_STRUCTS = {DP_K_PREPROC: PreprocParams, DP_K_ROWREDUCE: RowReduceParams, DP_K_GEMM: GemmParams,
                 DP_K_REGION: RegionDesc, DP_K_EMBEDDING: EmbeddingParams, DP_K_ATTENTION: AttentionParams,
                 DP_K_ROPE: RopeParams, DP_K_SPLITK: SplitKParams, DP_K_ARGMAX_KEYS: ArgmaxKeysParams,
                 DP_K_GEMM_SK: StreamKParams}

# (symbol, argtypes) of every exported function, in header order.
_VP = ctypes.c_void_p
EXPORTS = {
    "dp_version": [],
    "dp_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "dp_device_init": [ctypes.c_int],
    "dp_device_error": [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)],
    "dp_device_error_pending": [ctypes.c_int, ctypes.POINTER(ctypes.c_int)],
    "dp_set_wait_limit": [ctypes.c_int, ctypes.c_uint64],
    "dp_test_withhold_copies": [ctypes.c_int, ctypes.c_int],
    "dp_preproc": [ctypes.POINTER(PreprocParams), _VP, _VP, _VP],
    "dp_rowreduce": [ctypes.POINTER(RowReduceParams), _VP, _VP, _VP, _VP, _VP],
    "dp_gemm": [ctypes.POINTER(GemmParams), _VP, _VP, _VP, _VP, _VP, _VP],
    "dp_gemm_splitk_reduce": [ctypes.POINTER(SplitKParams), _VP, _VP, _VP, _VP, _VP],
    "dp_gemm_streamk_workspace": [ctypes.POINTER(GemmParams), ctypes.POINTER(ctypes.c_int64)],
    "dp_gemm_streamk": [ctypes.POINTER(StreamKParams), _VP, _VP, _VP, _VP, _VP, _VP, _VP],
    "dp_argmax_keys": [ctypes.POINTER(ArgmaxKeysParams), _VP, _VP, _VP],
    "dp_region": [ctypes.POINTER(RegionDesc), ctypes.POINTER(_VP), _VP],
    "dp_embedding": [ctypes.POINTER(EmbeddingParams), _VP, _VP, _VP, _VP],
    "dp_attention": [ctypes.POINTER(AttentionParams), _VP, _VP, _VP, _VP, _VP],
    "dp_rope": [ctypes.POINTER(RopeParams), _VP, _VP, _VP, _VP, _VP],
    "dp_program_create": [_VP, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(_VP)],
    "dp_program_bind": [_VP, ctypes.c_int, _VP, ctypes.c_size_t],
    "dp_program_run": [_VP, _VP],
    "dp_program_set_graph": [_VP, ctypes.c_int],
    "dp_program_arena_bytes": [_VP, ctypes.POINTER(ctypes.c_uint64)],
    "dp_program_destroy": [_VP],
    "dp_program_run_noalloc": [_VP, ctypes.c_size_t, ctypes.POINTER(_VP), ctypes.POINTER(ctypes.c_uint64),
                               ctypes.c_int, _VP],
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library; raises DevProcError if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = Path(os.environ.get("DEVPROC_B200_LIB", LIB_PATH))
                if not path.exists():
                    raise DevProcError(DP_ERR_STATE, f"native library {path} is missing; build it with "
                                                     "`python -m devproc_b200.csrc.build`")
                handle = ctypes.CDLL(str(path))
                for name, argtypes in EXPORTS.items():
                    fn = getattr(handle, name)
                    fn.argtypes = argtypes
                    fn.restype = ctypes.c_int
                _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().dp_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != DP_OK:
        raise DevProcError(status, f"{what}: {last_error()}" if what else last_error())


def device_init(device: int) -> None:
    check(lib().dp_device_init(device), "dp_device_init")


def device_error():
    """(code, info) of the device error word, which is then cleared (synchronises)."""
    code, info = ctypes.c_int(0), ctypes.c_int64(0)
    check(lib().dp_device_error(ctypes.byref(code), ctypes.byref(info)), "dp_device_error")
    return code.value, info.value


def device_error_pending(device: int) -> int:
    """DP_DEVERR_* code recorded on ``device`` since the last clear (no CUDA call;
    meaningful once the work that may have failed has been synchronised)."""
    code = ctypes.c_int(0)
    check(lib().dp_device_error_pending(device, ctypes.byref(code)), "dp_device_error_pending")
    return code.value


def raise_device_error(device: int, where: str) -> None:
    """Raise if a kernel on ``device`` recorded an error: IndexError for an
    out-of-range embedding id, DevProcError(DP_ERR_DEVICE) for a wait that
    gave up (with its site).  Reads and clears the word."""
    if device_error_pending(device) == DP_DEVERR_NONE:
        return
    import torch
    with torch.cuda.device(device):
        code, info = device_error()
    if code == DP_DEVERR_INDEX:
        raise IndexError(f"{where}: embedding id out of range at flat position {info}")
    if code == DP_DEVERR_TIMEOUT:
        raise DevProcError(DP_ERR_DEVICE, f"{where}: a bounded wait inside a kernel gave up (site {info}); "
                                          "the outputs of this run are incomplete")
    if code != DP_DEVERR_NONE:
        raise DevProcError(DP_ERR_DEVICE, f"{where}: device error {code} (info {info})")


def set_wait_limit(device: int, limit_ns: int) -> None:
    check(lib().dp_set_wait_limit(device, limit_ns), "dp_set_wait_limit")


def test_withhold_copies(device: int, enable: bool) -> None:
    check(lib().dp_test_withhold_copies(device, 1 if enable else 0), "dp_test_withhold_copies")


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def preproc(p: PreprocParams, x, out, stream=None) -> None:
    check(lib().dp_preproc(ctypes.byref(p), _ptr(x), _ptr(out), _stream(stream)), "dp_preproc")


def rowreduce(p: RowReduceParams, x, out, weight=None, bias=None, stream=None) -> None:
    check(lib().dp_rowreduce(ctypes.byref(p), _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), _stream(stream)),
          "dp_rowreduce")


def gemm(p: GemmParams, a, b, c, bias=None, residual=None, stream=None) -> None:
    check(lib().dp_gemm(ctypes.byref(p), _ptr(a), _ptr(b), _ptr(c), _ptr(bias), _ptr(residual),
                        _stream(stream)), "dp_gemm")


def gemm_splitk_reduce(p: SplitKParams, workspace, c, bias=None, residual=None, stream=None) -> None:
    check(lib().dp_gemm_splitk_reduce(ctypes.byref(p), _ptr(workspace), _ptr(c), _ptr(bias), _ptr(residual),
                                      _stream(stream)), "dp_gemm_splitk_reduce")


def gemm_streamk_workspace(p: GemmParams) -> int:
    """Bytes of stream-K workspace that always suffice for ``p`` on the current device."""
    n = ctypes.c_int64(0)
    check(lib().dp_gemm_streamk_workspace(ctypes.byref(p), ctypes.byref(n)), "dp_gemm_streamk_workspace")
    return n.value


def gemm_streamk(p: StreamKParams, a, b, c, workspace, bias=None, residual=None, stream=None) -> None:
    check(lib().dp_gemm_streamk(ctypes.byref(p), _ptr(a), _ptr(b), _ptr(c), _ptr(bias), _ptr(residual),
                                _ptr(workspace), _stream(stream)), "dp_gemm_streamk")


def argmax_keys(p: ArgmaxKeysParams, keys, out=None, stream=None) -> None:
    check(lib().dp_argmax_keys(ctypes.byref(p), _ptr(keys), _ptr(out), _stream(stream)), "dp_argmax_keys")


def region(d: RegionDesc, operands, stream=None) -> None:
    arr = (_VP * len(operands))(*[_ptr(o) for o in operands])
    check(lib().dp_region(ctypes.byref(d), arr, _stream(stream)), "dp_region")


def attention(p: AttentionParams, q, k, v, o, stream=None) -> None:
    check(lib().dp_attention(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _stream(stream)),
          "dp_attention")


def rope(p: RopeParams, x, cos, sin, out, stream=None) -> None:
    check(lib().dp_rope(ctypes.byref(p), _ptr(x), _ptr(cos), _ptr(sin), _ptr(out), _stream(stream)), "dp_rope")


def embedding(p: EmbeddingParams, ids, weight, out, stream=None) -> None:
    check(lib().dp_embedding(ctypes.byref(p), _ptr(ids), _ptr(weight), _ptr(out), _stream(stream)),
          "dp_embedding")


class NativeProgram:
    """Owner of one ``dp_program`` handle (arena + validated plan)."""

    def __init__(self, plan: bytes, device: int):
        h = _VP()
        check(lib().dp_program_create(plan, len(plan), device, ctypes.byref(h)), "dp_program_create")
        self._h = h
        self.device = device

    def bind(self, slot: int, ptr: int, nbytes: int) -> None:
        check(lib().dp_program_bind(self._h, slot, ptr, nbytes), f"dp_program_bind(slot {slot})")

    def run(self, stream) -> None:
        check(lib().dp_program_run(self._h, stream), "dp_program_run")

    def set_graph(self, enable: bool) -> None:
        check(lib().dp_program_set_graph(self._h, 1 if enable else 0), "dp_program_set_graph")

    def arena_bytes(self) -> int:
        v = ctypes.c_uint64(0)
        check(lib().dp_program_arena_bytes(self._h, ctypes.byref(v)), "dp_program_arena_bytes")
        return v.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            h, self._h = self._h, None
            if _lib is not None:
                _lib.dp_program_destroy(h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
