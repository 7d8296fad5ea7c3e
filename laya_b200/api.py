"""ctypes bindings of include/laya_b200.h and the host-side mirror of the reference's interfaces."""
import ctypes
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "liblaya_b200.so"

PRECISION_F32 = 0
PRECISION_Q8_0 = 1
F32, BF16, F16, I8, I32 = 0, 1, 2, 3, 4


# --------------------------------------------------------------------------------------------------- errors
class LayaError(RuntimeError):
    code = -1


class LayaArgumentError(LayaError, ValueError):      # ArgumentException
    code = 1


class LayaOutOfRangeError(LayaArgumentError, IndexError):   # ArgumentOutOfRangeException
    code = 2


class LayaNotSupportedError(LayaError, NotImplementedError):   # PlatformNotSupportedException
    code = 3


class LayaCudaError(LayaError):
    code = 4


class LayaNotFoundError(LayaError, KeyError):
    code = 5


class LayaDeviceTimeout(LayaError):
    code = 6


class LayaLibraryMissing(LayaError):
    pass


_ERRORS = {c.code: c for c in (LayaArgumentError, LayaOutOfRangeError, LayaNotSupportedError, LayaCudaError,
                               LayaNotFoundError, LayaDeviceTimeout)}


# --------------------------------------------------------------------------------------------------- library
class ModelDesc(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("intermediate", ctypes.c_int), ("layers", ctypes.c_int),
                ("heads", ctypes.c_int), ("vocab", ctypes.c_int), ("local_attention", ctypes.c_int),
                ("global_every", ctypes.c_int), ("layer_kinds", ctypes.POINTER(ctypes.c_int)),
                ("theta_global", ctypes.c_double), ("theta_local", ctypes.c_double), ("norm_eps", ctypes.c_float),
                ("head_layers", ctypes.c_int), ("n_act", ctypes.c_int), ("act_hidden", ctypes.c_int),
                ("precision", ctypes.c_int), ("max_tokens", ctypes.c_int), ("max_items", ctypes.c_int),
                ("max_markers", ctypes.c_int)]


def library_path():
    return os.path.join(HERE, _LIB_NAME)


_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGS = {
    "laya_last_error": (ctypes.c_char_p, []),
    "laya_version": (ctypes.c_char_p, []),
    "laya_ctx_create": (_I, [ctypes.POINTER(ModelDesc), _I, ctypes.POINTER(_P)]),
    "laya_ctx_destroy": (_I, [_P]),
    "laya_ctx_set_stream": (_I, [_P, _P]),
    "laya_ctx_get_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_ctx_synchronize": (_I, [_P]),
    "laya_ctx_launches": (_I, [_P, ctypes.POINTER(ctypes.c_longlong)]),
    "laya_ctx_set_profiling": (_I, [_P, _I]),
    "laya_ctx_profile": (_I, [_P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(ctypes.c_longlong)]),
    "laya_upload_tensor": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P]),
    "laya_upload_q8_0": (_I, [_P, ctypes.c_char_p, _P, _P, _I, _I]),
    "laya_download_tensor": (_I, [_P, ctypes.c_char_p, _P, ctypes.c_int64]),
    "laya_q8_0_linear": (_I, [_P, ctypes.c_char_p, _P, _I, _I, _P, _P, _I]),
    "laya_q8_0_linear_device": (_I, [_P, ctypes.c_char_p, _P, _I, _I, _P, _P, _I]),
    "laya_q8_0_quantize_activations_device": (_I, [_P, _P, _I, _I, _I, _P, _P, _I]),
    "laya_q8_0_quantize_weights_device": (_I, [_P, _P, _I, _I, _P, _P, _I]),
    "laya_q8_0_gemm_device": (_I, [_P, _P, _P, _I, _I, _P, _P, _I, _I, _I, _P, _P, _I]),
    "laya_q8_0_gemm_fused_device": (_I, [_P, _I, _P, _P, _I, _I, _P, _P, _I, _I, _I, _P, _P, _I, _P, _P, _I]),
    "laya_pack_q8_0": (_I, [_P, ctypes.c_char_p, _I, _P, _I, _I]),
    "laya_q8_0_linear_noalloc": (_I, [_P, _I, _I, _P, _P, _I, _I, _I, _P, _P, _I, _P]),
    "laya_mma_peak": (_I, [_I, _I, _I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "laya_gemm_bf16_device": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _I, _P, _I]),
    "laya_gemm_bf16_split_device": (_I, [_P, _I, _I, _I, _P, _P, _I, _I, _P, _P, _I, _I, _P, _I, _P, _I]),
    "laya_decision_forward": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _P]),
    "laya_decision_forward_device": (_I, [_P, _P, _P, _P, _I, _I, _P, _P, _I, _P, _P]),
    "laya_encoder_forward": (_I, [_P, _P, _P, _I, _P]),
    "laya_record_enable": (_I, [_P, _I]),
    "laya_record_get": (_I, [_P, ctypes.c_char_p, _P, ctypes.c_int64]),
    "laya_encoder_layer": (_I, [_P, _I, _P, _P, _I]),
    # include/laya_train.h
    "laya_trainer_create": (_I, [ctypes.POINTER(ModelDesc), _P, _I, ctypes.POINTER(_P)]),
    "laya_trainer_destroy": (_I, [_P]),
    "laya_trainer_set_stream": (_I, [_P, _P]),
    "laya_trainer_get_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_trainer_synchronize": (_I, [_P]),
    "laya_trainer_upload": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P]),
    "laya_trainer_download": (_I, [_P, ctypes.c_char_p, _P, ctypes.c_int64]),
    "laya_trainer_download_grad": (_I, [_P, ctypes.c_char_p, _P, ctypes.c_int64]),
    "laya_trainer_param_count": (_I, [_P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "laya_trainer_param_info": (_I, [_P, _I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_int64),
                                     ctypes.POINTER(ctypes.c_int64)]),
    "laya_batch_create": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_batch_destroy": (_I, [_P]),
    "laya_batch_set": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I]),
    "laya_batch_shape": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "laya_train_forward": (_I, [_P, _P, _I, ctypes.c_uint64, _P]),
    "laya_train_objective": (_I, [_P, _P, _P, _P, _P]),
    "laya_train_backward": (_I, [_P, _P, _P]),
    "laya_train_set_lr": (_I, [_P, _P, _I]),
    "laya_train_clip_and_step": (_I, [_P, ctypes.c_double, _P]),
    "laya_train_zero_grads": (_I, [_P]),
    "laya_train_steps": (_I, [_P, ctypes.POINTER(ctypes.c_int64)]),
    "laya_trainer_launches": (_I, [_P, ctypes.POINTER(ctypes.c_longlong)]),
    "laya_trainer_set_profiling": (_I, [_P, _I]),
    "laya_trainer_profile": (_I, [_P, _I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_longlong)]),
    "laya_fit_temperatures": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "laya_train_calibrate": (_I, [_P, _P, _I, _I, _P]),
    "laya_trainer_save_checkpoint": (_I, [_P, ctypes.c_char_p, _I]),
    "laya_trainer_restore_checkpoint": (_I, [_P, ctypes.c_char_p]),
    "laya_comm_unique_id": (_I, [_P]),
    "laya_train_comm_init": (_I, [_P, _P, _I, _I]),
    # include/laya_decoder.h
    "laya_decoder_create": (_I, [_P, _I, ctypes.POINTER(_P)]),
    "laya_decoder_destroy": (_I, [_P]),
    "laya_decoder_set_stream": (_I, [_P, _P]),
    "laya_decoder_get_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_decoder_synchronize": (_I, [_P]),
    "laya_decoder_upload": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_int64), _I, _P]),
    "laya_decoder_upload_q8_0": (_I, [_P, ctypes.c_char_p, _P, _P, _I, _I]),
    "laya_decoder_missing": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(_I)]),
    "laya_decoder_forward": (_I, [_P, _P, _P, _I, _P, _I, _P, _P]),
    "laya_decoder_forward_device": (_I, [_P, _P, _P, _I, _P, _I, _P, _P]),
    "laya_decoder_logits": (_I, [_P, _P, _I, _P, _I, _P]),
    "laya_decoder_layer": (_I, [_P, _I, _P, _P, _I, _P]),
    "laya_decoder_state_create": (_I, [_P, _I, ctypes.POINTER(_P)]),
    "laya_decoder_state_destroy": (_I, [_P]),
    "laya_decoder_state_length": (_I, [_P, ctypes.POINTER(_I)]),
    "laya_decoder_state_bytes": (_I, [_P, ctypes.POINTER(ctypes.c_int64)]),
    "laya_decoder_state_clone": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_decoder_state_save": (_I, [_P, ctypes.POINTER(_P)]),
    "laya_decoder_state_rewind": (_I, [_P, _P]),
    "laya_decoder_mark_destroy": (_I, [_P]),
    "laya_decoder_forward_states": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P]),
    "laya_decoder_set_chunked_delta_rule": (_I, [_P, _I]),
    "laya_decoder_record_enable": (_I, [_P, _I]),
    "laya_decoder_record_get": (_I, [_P, ctypes.c_char_p, _P, ctypes.c_int64]),
    "laya_decoder_launches": (_I, [_P, ctypes.POINTER(ctypes.c_longlong)]),
    "laya_decoder_set_profiling": (_I, [_P, _I]),
    "laya_decoder_profile": (_I, [_P, _I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_longlong)]),
}


def lib():
    """The loaded liblaya_b200.so (raises LayaLibraryMissing if it was not built)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not os.path.exists(path):
            raise LayaLibraryMissing(f"{path} is missing: build it with `python -m laya_b200.build`")
        L = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        msg = lib().laya_last_error().decode("utf-8", "replace")
        raise _ERRORS.get(rc, LayaError)(msg)


def _np_ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def base_desc(**kw) -> ModelDesc:
    """ModernBERT-base geometry (22 layers, h 768, 12×64, I 1152, vocab 50368) with a Laya decision head."""
    d = dict(hidden=768, intermediate=1152, layers=22, heads=12, vocab=50368, local_attention=128, global_every=3,
             theta_global=160000.0, theta_local=10000.0, norm_eps=1e-5, head_layers=2, n_act=2, act_hidden=256,
             precision=PRECISION_Q8_0, max_tokens=32768, max_items=256, max_markers=4096)
    d.update(kw)
    kinds = d.pop("layer_kinds", None)
    desc = ModelDesc(**d)
    if kinds is not None:
        arr = (ctypes.c_int * len(kinds))(*kinds)
        desc.layer_kinds = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int))
        desc._kinds_keepalive = arr
    return desc


# --------------------------------------------------------------------------------------------------- context
class Context:
    """A device context (laya_ctx): weights by name, workspaces, stream."""

    def __init__(self, desc: ModelDesc, device: int = 0):
        self.desc = desc
        h = ctypes.c_void_p()
        check(lib().laya_ctx_create(ctypes.byref(desc), device, ctypes.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_handle: Optional[int]):
        """Launch on this cudaStream_t from now on (0 / None: CUDA's legacy default stream, torch's default)."""
        check(lib().laya_ctx_set_stream(self.handle, stream_handle or None))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().laya_ctx_get_stream(self.handle, ctypes.byref(s)))
        return s.value or 0

    def synchronize(self):
        check(lib().laya_ctx_synchronize(self.handle))

    def launches(self) -> int:
        n = ctypes.c_longlong()
        check(lib().laya_ctx_launches(self.handle, ctypes.byref(n)))
        return n.value

    def set_profiling(self, enabled: bool):
        check(lib().laya_ctx_set_profiling(self.handle, 1 if enabled else 0))

    def profile(self) -> Tuple[float, float, int]:
        ms, ops, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_longlong()
        check(lib().laya_ctx_profile(self.handle, ctypes.byref(ms), ctypes.byref(ops), ctypes.byref(n)))
        return ms.value, ops.value, n.value

    def upload(self, name: str, array: np.ndarray):
        a = np.ascontiguousarray(array)
        if a.dtype == np.float32:
            dt = F32
        elif a.dtype == np.float16:
            dt = F16
        else:
            a = a.astype(np.float32)
            dt = F32
        shape = (ctypes.c_int64 * a.ndim)(*a.shape)
        check(lib().laya_upload_tensor(self.handle, name.encode(), dt, shape, a.ndim, _np_ptr(a)))

    def upload_bf16_bits(self, name: str, bits: np.ndarray):
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        shape = (ctypes.c_int64 * a.ndim)(*a.shape)
        check(lib().laya_upload_tensor(self.handle, name.encode(), BF16, shape, a.ndim, _np_ptr(a)))

    def upload_q8_0(self, name: str, q: np.ndarray, d_fp16: np.ndarray):
        q = np.ascontiguousarray(q, dtype=np.int8)
        d = np.ascontiguousarray(d_fp16, dtype=np.float16).view(np.uint16)
        N, K = q.shape
        check(lib().laya_upload_q8_0(self.handle, name.encode(), _np_ptr(q), _np_ptr(d), N, K))

    def download(self, name: str, shape) -> np.ndarray:
        out = np.zeros(shape, np.float32)
        check(lib().laya_download_tensor(self.handle, name.encode(), _np_ptr(out), out.size))
        return out

    def record(self, enabled: bool):
        check(lib().laya_record_enable(self.handle, 1 if enabled else 0))

    def recorded(self, name: str, shape) -> np.ndarray:
        out = np.zeros(shape, np.float32)
        check(lib().laya_record_get(self.handle, name.encode(), _np_ptr(out), out.size))
        return out


# --------------------------------------------------------------------------------------------------- ILinear
class PackedMatrixQ8_0:
    """A Q8_0 projection (PackedMatrixQ8_0, Base/Numerics/PackedMatrixQ8_0.cs:108-246) living in a Context.

    Construct from a PyTorch-layout [out, in] fp32 weight (quantized on the device by ggml's weight quantizer,
    PackedMatrixQ8_0.cs:168-173) or from Q8_0 codes + fp16 scales.  `multiply` is ILinear.Multiply.
    """

    def __init__(self, ctx: Context, name: str, weight: Optional[np.ndarray] = None,
                 q: Optional[np.ndarray] = None, d_fp16: Optional[np.ndarray] = None):
        self.ctx, self.name = ctx, name
        if weight is not None:
            w = np.ascontiguousarray(weight)
            if w.dtype == np.uint16:          # raw bf16 bit patterns, as the bf16 constructor takes them
                dt = BF16
            else:
                w = _f32(w)
                dt = F32
            self.out_features, self.in_features = w.shape
            check(lib().laya_pack_q8_0(ctx.handle, name.encode(), dt, _np_ptr(w), w.shape[0], w.shape[1]))
        else:
            ctx.upload_q8_0(name, q, d_fp16)
            self.out_features, self.in_features = q.shape

    def multiply(self, input: np.ndarray, rows: int, input_stride: Optional[int] = None,
                 bias: Optional[np.ndarray] = None, output: Optional[np.ndarray] = None,
                 output_stride: Optional[int] = None) -> np.ndarray:
        input_stride = self.in_features if input_stride is None else input_stride
        output_stride = self.out_features if output_stride is None else output_stride
        x = _f32(input).reshape(-1)
        if rows > 0 and x.size < (rows - 1) * input_stride + self.in_features:
            raise LayaArgumentError("input is too small")
        if output is None:
            output = np.zeros(max(rows, 1) * output_stride, np.float32)
        if rows > 0 and output.size < (rows - 1) * output_stride + self.out_features:
            raise LayaArgumentError("output is too small")
        b = None if bias is None or len(bias) == 0 else _f32(bias)
        if b is not None and b.size < self.out_features:
            raise LayaArgumentError("bias is too small")
        check(lib().laya_q8_0_linear(self.ctx.handle, self.name.encode(), _np_ptr(x), rows, input_stride,
                                     _np_ptr(b), output.ctypes.data_as(ctypes.c_void_p), output_stride))
        return output

    def dequantize(self) -> np.ndarray:
        """Every column's q·d (PackedMatrixQ8_0.Dequantize, PackedMatrixQ8_0.cs:209-218), as [out, in]."""
        return self.ctx.download(self.name, (self.out_features, self.in_features))


class Q8_0:
    """The two ggml quantizers and the product on device buffers (Q8_0, Base/Numerics/PackedMatrixQ8_0.cs:15-72).

    Pointers are device addresses (ints), e.g. torch tensors' data_ptr().  Codes are fp16 values equal to the integer
    codes (-127..127); block scales are fp32 [blocks, stride].
    """
    BlockSize = 32

    @staticmethod
    def quantize_activations(ctx: Context, x_ptr: int, rows: int, stride: int, features: int, q_ptr: int,
                             d_ptr: int, ldd: int):
        check(lib().laya_q8_0_quantize_activations_device(ctx.handle, x_ptr, rows, stride, features, q_ptr, d_ptr,
                                                          ldd))

    @staticmethod
    def quantize_weights(ctx: Context, w_ptr: int, n: int, k: int, q_ptr: int, d_ptr: int, ldd: int):
        check(lib().laya_q8_0_quantize_weights_device(ctx.handle, w_ptr, n, k, q_ptr, d_ptr, ldd))

    @staticmethod
    def gemm(ctx: Context, qx_ptr, dx_ptr, ldx, m, qw_ptr, dw_ptr, ldw, n, k, bias_ptr, out_ptr, ldo):
        check(lib().laya_q8_0_gemm_device(ctx.handle, qx_ptr, dx_ptr, ldx, m, qw_ptr, dw_ptr, ldw, n, k, bias_ptr,
                                          out_ptr, ldo))

    STORE, RESIDUAL, GEGLU, RELU, SWIGLU = 0, 1, 2, 3, 4

    @staticmethod
    def gemm_fused(ctx: Context, epilogue, qx_ptr, dx_ptr, ldx, m, qw_ptr, dw_ptr, ldw, n, k, bias_ptr, out_ptr, ldo,
                   qout_ptr, qscale_ptr, ldqs):
        check(lib().laya_q8_0_gemm_fused_device(ctx.handle, epilogue, qx_ptr, dx_ptr, ldx, m, qw_ptr, dw_ptr, ldw, n,
                                                k, bias_ptr, out_ptr, ldo, qout_ptr, qscale_ptr, ldqs))


# --------------------------------------------------------------------------------------------------- model
@dataclass
class BatchItem:
    """DecisionModel.BatchItem (Laya/Models/DecisionModel.cs:107)."""
    token_ids: Sequence[int]
    marker_positions: Sequence[int]
    type: int


@dataclass
class DecisionOutput:
    """DecisionOutput (Laya/Models/DecisionModel.cs:10)."""
    option_logits: np.ndarray
    action_probabilities: np.ndarray


class DecisionModel:
    """The decision model's batched inference forward on the device (DecisionModel + ModernBertEncoder).

    `weights` maps safetensors names to arrays; `q8` maps projection names to (codes int8 [N, K], scales fp16
    [N, K/32]) for checkpoints already in Q8_0.  In a PRECISION_Q8_0 context projections given as floats are quantized
    on the device; in a PRECISION_F32 context they are kept as bf16 hi/lo parts (the lo part dropped when every weight
    is a bf16 value) and the forward runs the fp32-accurate split products (PackedMatrix, DecisionModel.cs:50-99).
    """

    def __init__(self, desc: ModelDesc, weights: Dict[str, np.ndarray], q8: Optional[Dict] = None, device: int = 0):
        self.desc = desc
        self.ctx = Context(desc, device)
        for name, arr in weights.items():
            if q8 and name in q8:
                continue
            if name == "temperature":
                continue
            self.ctx.upload(name, arr)
        for name, (q, d) in (q8 or {}).items():
            self.ctx.upload_q8_0(name, q, d)

    @staticmethod
    def pack(items: List[BatchItem]):
        ids = _i32(np.concatenate([np.asarray(it.token_ids, np.int64) for it in items])) if items else _i32([])
        seg_len = _i32([len(it.token_ids) for it in items])
        qtype = _i32([it.type for it in items])
        counts = _i32([len(it.marker_positions) for it in items])
        markers = _i32(np.concatenate([np.asarray(it.marker_positions, np.int64) for it in items])
                       if items and counts.sum() else np.zeros(1))
        return ids, seg_len, qtype, counts, markers

    def forward(self, items: List[BatchItem]) -> List[DecisionOutput]:
        """DecisionModel.Forward (Laya/Models/DecisionModel.cs:128-169)."""
        if not items:
            return []
        ids, seg_len, qtype, counts, markers = self.pack(items)
        logits = np.zeros(max(1, int(counts.sum())), np.float32)
        act = np.zeros(len(items) * self.desc.n_act, np.float32)
        check(lib().laya_decision_forward(self.ctx.handle, _np_ptr(ids), _np_ptr(seg_len), _np_ptr(qtype),
                                          len(items), _np_ptr(counts), _np_ptr(markers), _np_ptr(logits),
                                          _np_ptr(act)))
        out, m = [], 0
        for i, it in enumerate(items):
            k = len(it.marker_positions)
            out.append(DecisionOutput(logits[m:m + k].copy(), act[i * self.desc.n_act:(i + 1) * self.desc.n_act].copy()))
            m += k
        return out

    def encoder_forward(self, token_ids: Sequence[np.ndarray]) -> np.ndarray:
        """ModernBertEncoder.Forward over concatenated segments: final hidden states [T, hidden]."""
        ids = _i32(np.concatenate([np.asarray(t, np.int64) for t in token_ids]))
        seg_len = _i32([len(t) for t in token_ids])
        out = np.zeros((ids.size, self.desc.hidden), np.float32)
        check(lib().laya_encoder_forward(self.ctx.handle, _np_ptr(ids), _np_ptr(seg_len), len(seg_len),
                                         _np_ptr(out)))
        return out

    def encoder_layer(self, layer: int, hidden: np.ndarray, seg_len: Sequence[int]) -> np.ndarray:
        """Runs one encoder layer on given hidden states (teacher forcing for per-layer parity)."""
        h = _f32(hidden).copy()
        sl = _i32(seg_len)
        check(lib().laya_encoder_layer(self.ctx.handle, layer, _np_ptr(h), _np_ptr(sl), len(sl)))
        return h


# --------------------------------------------------------------------------------------------------- training
MAX_TEMPERATURE_BUCKETS = 12


class TemperatureFitDesc(ctypes.Structure):
    """laya_temperature_fit (include/laya_train.h): TemperatureFit (Laya.Training/TemperatureFitting.cs:10-11)."""
    _fields_ = [("by_type", ctypes.c_float * 3), ("n_buckets", ctypes.c_int),
                ("bucket", (ctypes.c_char * 16) * MAX_TEMPERATURE_BUCKETS),
                ("bucket_count", ctypes.c_int * MAX_TEMPERATURE_BUCKETS),
                ("bucket_fitted", ctypes.c_int * MAX_TEMPERATURE_BUCKETS),
                ("bucket_temperature", ctypes.c_float * MAX_TEMPERATURE_BUCKETS)]

    def result(self):
        """(by_type [choice, score, noul], {bucket: temperature} of the fitted buckets, {bucket: samples})."""
        names = [self.bucket[i].value.decode() for i in range(self.n_buckets)]
        fitted = {n: float(self.bucket_temperature[i]) for i, n in enumerate(names) if self.bucket_fitted[i]}
        return [float(v) for v in self.by_type], fitted, {n: int(self.bucket_count[i]) for i, n in enumerate(names)}


def fit_temperatures(samples, minimum_bucket_samples: int = 30):
    """TemperatureFitting.Fit on host samples [(question_type, logits, target)] through the C ABI."""
    q = _i32([s[0] for s in samples])
    k = _i32([len(s[1]) for s in samples])
    z = _f32(np.concatenate([np.asarray(s[1], np.float32) for s in samples]) if samples else np.zeros(0))
    t = _f32(np.concatenate([np.asarray(s[2], np.float32) for s in samples]) if samples else np.zeros(0))
    out = TemperatureFitDesc()
    check(lib().laya_fit_temperatures(_np_ptr(q), _np_ptr(k), _np_ptr(z), _np_ptr(t), len(samples),
                                      minimum_bucket_samples, ctypes.byref(out)))
    return out.result()


class TrainDesc(ctypes.Structure):
    """laya_train_desc (include/laya_train.h): TrainerOptions + AdamW settings (Trainer.cs:16-58)."""
    _fields_ = [("trainable_encoder_layers", ctypes.c_int), ("head_dropout", ctypes.c_float),
                ("beta1", ctypes.c_double), ("beta2", ctypes.c_double), ("eps", ctypes.c_double),
                ("weight_decay", ctypes.c_double), ("encoder_lr", ctypes.c_double), ("head_lr", ctypes.c_double),
                ("max_segment", ctypes.c_int), ("grad_accumulation", ctypes.c_int), ("forward_mode", ctypes.c_int)]


FORWARD_ACCURATE = 0   # fp32-accurate forward from bf16 hi/lo tensor-core products (the fp32 reference path)
FORWARD_BF16 = 1       # bf16-operand forward (torch.autocast(bfloat16) numerics)


class RlcdDesc(ctypes.Structure):
    """laya_rlcd_desc: RlcdObjective settings (RlcdObjective.cs:31-35) + sigma and gradient scale."""
    _fields_ = [("groups", ctypes.c_int), ("sigma", ctypes.c_double), ("scale", ctypes.c_double),
                ("spherical_weight", ctypes.c_double), ("rps_weight", ctypes.c_double),
                ("cross_entropy_weight", ctypes.c_double)]


def train_desc(**kw) -> TrainDesc:
    """Trainer defaults (TrainerOptions: encoder 2.5e-5, head 1e-4, wd 0.01, dropout 0.1; AdamW 0.9/0.999/1e-8)."""
    d = dict(trainable_encoder_layers=-1, head_dropout=0.1, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01,
             encoder_lr=2.5e-5, head_lr=1e-4, max_segment=0, grad_accumulation=1, forward_mode=FORWARD_ACCURATE)
    d.update(kw)
    return TrainDesc(**d)


@dataclass
class TrainingItem:
    """TrainingItem (Laya.Training): token ids, option marker positions, question type, soft target per option."""
    token_ids: np.ndarray
    marker_positions: np.ndarray
    question_type: int
    target: Optional[np.ndarray] = None

    @property
    def options(self) -> int:
        return len(self.marker_positions)


class Batch:
    """A batch resident on the device (laya_batch)."""

    def __init__(self, trainer: "Trainer"):
        self.trainer = trainer
        h = ctypes.c_void_p()
        check(lib().laya_batch_create(trainer.handle, ctypes.byref(h)))
        self.handle = h

    def set(self, items: List[TrainingItem], draws: Optional[np.ndarray] = None):
        """draws: standard normals [groups, options] in item order (RlcdObjective's supplied-draws overload)."""
        ids = _i32(np.concatenate([np.asarray(it.token_ids, np.int64) for it in items]))
        seg_len = _i32([len(it.token_ids) for it in items])
        qtype = _i32([it.question_type for it in items])
        counts = _i32([it.options for it in items])
        markers = _i32(np.concatenate([np.asarray(it.marker_positions, np.int64) for it in items]))
        tg = [np.zeros(it.options, np.float32) if it.target is None else np.asarray(it.target, np.float32)
              for it in items]
        targets = _f32(np.concatenate(tg))
        groups = 0
        dr = None
        if draws is not None:
            dr = np.ascontiguousarray(draws, dtype=np.float64)
            groups = dr.shape[0]
            if dr.shape[1] != int(counts.sum()):
                raise LayaArgumentError("draws must be [groups, options]")
        check(lib().laya_batch_set(self.trainer.handle, self.handle, _np_ptr(ids), _np_ptr(seg_len), _np_ptr(qtype),
                                   len(items), _np_ptr(counts), _np_ptr(markers), _np_ptr(targets), _np_ptr(dr),
                                   groups))
        self.counts = counts
        self._keep = (ids, seg_len, qtype, counts, markers, targets, dr)   # pinned staging copies them; keep anyway
        return self

    def shape(self):
        t, n, m = _I(), _I(), _I()
        check(lib().laya_batch_shape(self.handle, ctypes.byref(t), ctypes.byref(n), ctypes.byref(m)))
        return t.value, n.value, m.value

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_batch_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Trainer:
    """The fine-tuning step on the device (laya_trainer): TrainableDecisionModel + RlcdObjective + AdamW."""

    def __init__(self, desc: ModelDesc, tdesc: Optional[TrainDesc] = None, device: int = 0):
        self.desc = desc
        self.tdesc = tdesc or train_desc()
        h = ctypes.c_void_p()
        check(lib().laya_trainer_create(ctypes.byref(desc), ctypes.byref(self.tdesc), device, ctypes.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_trainer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # parameters
    def names(self) -> List[Tuple[str, int, int]]:
        out = []
        i = 0
        while True:
            nm, r, c = ctypes.c_char_p(), ctypes.c_int64(), ctypes.c_int64()
            rc = lib().laya_trainer_param_info(self.handle, i, ctypes.byref(nm), ctypes.byref(r), ctypes.byref(c))
            if rc != 0:
                break
            out.append((nm.value.decode(), r.value, c.value))
            i += 1
        return out

    def upload(self, name: str, array: np.ndarray, dtype: int = F32):
        a = np.ascontiguousarray(array, dtype=np.float32 if dtype == F32 else np.uint16)
        shape = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
        check(lib().laya_trainer_upload(self.handle, name.encode(), dtype, shape, a.ndim, _np_ptr(a)))

    def load(self, weights: Dict[str, np.ndarray]):
        for k, v in weights.items():
            self.upload(k, v)

    def download(self, name: str, shape) -> np.ndarray:
        out = np.zeros(shape, np.float32)
        check(lib().laya_trainer_download(self.handle, name.encode(), _np_ptr(out), out.size))
        return out

    def calibrate(self, batches: Sequence["Batch"], minimum_bucket_samples: int = 30):
        """Trainer.Calibrate: forward-only passes over the batches, then TemperatureFitting.Fit on their logits."""
        arr = (ctypes.c_void_p * max(1, len(batches)))(*[b.handle for b in batches])
        out = TemperatureFitDesc()
        check(lib().laya_train_calibrate(self.handle, arr, len(batches), minimum_bucket_samples, ctypes.byref(out)))
        return out.result()

    def save_checkpoint(self, path: str, with_optimizer: bool = True):
        """TrainableDecisionModel.Save's model.safetensors (parameters in their uploaded dtypes), plus AdamW's state."""
        check(lib().laya_trainer_save_checkpoint(self.handle, os.fsencode(path), 1 if with_optimizer else 0))

    def restore_checkpoint(self, path: str):
        check(lib().laya_trainer_restore_checkpoint(self.handle, os.fsencode(path)))

    def gradient(self, name: str, shape) -> np.ndarray:
        out = np.zeros(shape, np.float32)
        check(lib().laya_trainer_download_grad(self.handle, name.encode(), _np_ptr(out), out.size))
        return out

    def param_count(self) -> Tuple[int, int]:
        a, b = ctypes.c_int64(), ctypes.c_int64()
        check(lib().laya_trainer_param_count(self.handle, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def batch(self, items: List[TrainingItem], draws: Optional[np.ndarray] = None) -> Batch:
        return Batch(self).set(items, draws)

    # the step
    def forward(self, batch: Batch, training: bool = False, seed: int = 0, fetch: bool = True):
        """TrainableDecisionModel.Forward: option logits per item (device-resident tape kept for backward)."""
        _, _, m = batch.shape()
        logits = np.zeros(max(1, m), np.float32) if fetch else None
        check(lib().laya_train_forward(self.handle, batch.handle, int(training), ctypes.c_uint64(seed & (2**64 - 1)),
                                       _np_ptr(logits)))
        if not fetch:
            return None
        out, o = [], 0
        for k in batch.counts:
            out.append(logits[o:o + k].copy())
            o += k
        return out

    def objective(self, batch: Batch, sigma: float, groups: int = 4, scale: float = 1.0, spherical_weight=0.75,
                  rps_weight=1.0, cross_entropy_weight=1.0, fetch: bool = True):
        """RlcdObjective.Compute with the batch's draws: ((loss, policy, cross-entropy, mean reward), dlogits per item)."""
        o = RlcdDesc(groups, sigma, scale, spherical_weight, rps_weight, cross_entropy_weight)
        res = np.zeros(4, np.float64) if fetch else None
        d = np.zeros(max(1, int(batch.counts.sum())), np.float32) if fetch else None
        check(lib().laya_train_objective(self.handle, batch.handle, ctypes.byref(o), _np_ptr(res), _np_ptr(d)))
        if res is None:
            return None
        grads, k0 = [], 0
        for k in batch.counts:
            grads.append(d[k0:k0 + k].copy())
            k0 += k
        return tuple(float(x) for x in res), grads

    def backward(self, batch: Batch, dlogits: Optional[Sequence[np.ndarray]] = None):
        """TrainableDecisionModel.Backward: accumulates gradients; dlogits per item, or None for the objective's."""
        d = None if dlogits is None else _f32(np.concatenate([np.asarray(x, np.float32) for x in dlogits]))
        check(lib().laya_train_backward(self.handle, batch.handle, _np_ptr(d)))

    def set_lr(self, encoder_lr: float, head_lr: float):
        lr = np.array([encoder_lr, head_lr], np.float64)
        check(lib().laya_train_set_lr(self.handle, _np_ptr(lr), 2))

    def clip_and_step(self, max_norm: float = 1.0, fetch_norm: bool = True) -> Optional[float]:
        norm = np.zeros(1, np.float64) if fetch_norm else None
        check(lib().laya_train_clip_and_step(self.handle, max_norm, _np_ptr(norm)))
        return None if norm is None else float(norm[0])

    def zero_grads(self):
        check(lib().laya_train_zero_grads(self.handle))

    def synchronize(self):
        check(lib().laya_trainer_synchronize(self.handle))

    def set_stream(self, stream_handle: Optional[int]):
        check(lib().laya_trainer_set_stream(self.handle, ctypes.c_void_p(stream_handle or 0)))

    def steps(self) -> int:
        s = ctypes.c_int64()
        check(lib().laya_train_steps(self.handle, ctypes.byref(s)))
        return s.value

    def launches(self) -> int:
        n = ctypes.c_longlong()
        check(lib().laya_trainer_launches(self.handle, ctypes.byref(n)))
        return n.value

    def set_profiling(self, enabled: bool):
        check(lib().laya_trainer_set_profiling(self.handle, int(enabled)))

    PRODUCTS, ATTENTION_FWD, ATTENTION_BWD = 0, 1, 2

    def profile(self, kind: int) -> Tuple[float, float, int]:
        """(milliseconds, algorithmic FLOPs, launches) of one kernel kind since the last call."""
        ms, fl, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_longlong()
        check(lib().laya_trainer_profile(self.handle, kind, ctypes.byref(ms), ctypes.byref(fl), ctypes.byref(n)))
        return ms.value, fl.value, n.value

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().laya_comm_unique_id(buf))
        return buf.raw

    def comm_init(self, uid: bytes, rank: int, world: int):
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        check(lib().laya_train_comm_init(self.handle, buf, rank, world))


# --------------------------------------------------------------------------------------------------- Mica decoder
DECODER_LINEAR, DECODER_FULL = 0, 1


class DecoderDesc(ctypes.Structure):
    """laya_decoder_desc: Qwen35Config (Mica/Models/Qwen35Config.cs:60-130) plus the capacity of one forward."""
    _fields_ = [("hidden", ctypes.c_int), ("intermediate", ctypes.c_int), ("layers", ctypes.c_int),
                ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("layer_kinds", ctypes.POINTER(ctypes.c_int32)),
                ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("rope_theta", ctypes.c_double), ("rotary_dim", ctypes.c_int), ("lin_k_heads", ctypes.c_int),
                ("lin_v_heads", ctypes.c_int), ("lin_k_dim", ctypes.c_int), ("lin_v_dim", ctypes.c_int),
                ("conv_kernel", ctypes.c_int), ("max_tokens", ctypes.c_int), ("max_seqs", ctypes.c_int)]


def decoder_desc(kinds: Sequence[str], **kw) -> DecoderDesc:
    """A DecoderDesc from layer kinds ("linear" | "full") and Qwen35Config fields; defaults are config 5's geometry
    (h 2560, I 9216, vocab 151936, 16 q / 4 kv heads × 128 with a quarter rotated at θ 1e7, DeltaNet 16 × 128 key and
    value heads, conv 4)."""
    d = dict(hidden=2560, intermediate=9216, vocab=151936, eps=1e-6, heads=16, kv_heads=4, head_dim=128,
             rope_theta=1e7, rotary_dim=32, lin_k_heads=16, lin_v_heads=16, lin_k_dim=128, lin_v_dim=128,
             conv_kernel=4, max_tokens=16384, max_seqs=8)
    d.update(kw)
    arr = (ctypes.c_int32 * max(1, len(kinds)))(*[DECODER_FULL if k == "full" else DECODER_LINEAR for k in kinds])
    desc = DecoderDesc(layers=len(kinds), **d)
    desc.layer_kinds = ctypes.cast(arr, ctypes.POINTER(ctypes.c_int32))
    desc._kinds_keepalive = arr
    return desc


class Qwen35Mark:
    """Qwen35State.Mark (Qwen35Model.cs:158-181): a saved point of a state; close() is Dispose."""

    def __init__(self, handle, length: int):
        self.handle = handle
        self.length = length

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_decoder_mark_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Qwen35State:
    """Qwen35State (Qwen35Model.cs:38-197) in device memory: what the decoder remembers of the tokens read so far.
    Length, Bytes, Clone, Save / Rewind; close() is Dispose."""

    def __init__(self, handle):
        self.handle = handle

    @property
    def length(self) -> int:
        n = ctypes.c_int()
        check(lib().laya_decoder_state_length(self.handle, ctypes.byref(n)))
        return n.value

    @property
    def bytes(self) -> int:
        n = ctypes.c_int64()
        check(lib().laya_decoder_state_bytes(self.handle, ctypes.byref(n)))
        return n.value

    def clone(self) -> "Qwen35State":
        h = ctypes.c_void_p()
        check(lib().laya_decoder_state_clone(self.handle, ctypes.byref(h)))
        return Qwen35State(h)

    def save(self) -> Qwen35Mark:
        h = ctypes.c_void_p()
        check(lib().laya_decoder_state_save(self.handle, ctypes.byref(h)))
        return Qwen35Mark(h, self.length)

    def rewind(self, mark: Qwen35Mark):
        check(lib().laya_decoder_state_rewind(self.handle, mark.handle))

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_decoder_state_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Qwen35Sequence:
    """Qwen35Sequence (Qwen35Model.cs:199-221): tokens read after what `state` holds; `readout`; `checkpoints`
    (token counts, ascending) after which to snapshot the state.  A forward sets `hidden`, `logits` and
    `snapshots` (new states owned by the caller)."""

    def __init__(self, tokens, state: Qwen35State, readout: bool = True, checkpoints: Optional[Sequence[int]] = None):
        self.tokens = np.asarray(tokens, np.int64)
        self.state = state
        self.readout = readout
        self.checkpoints = list(checkpoints or [])
        self.hidden = None
        self.logits = None
        self.snapshots: List[Qwen35State] = []


class Qwen35Model:
    """The Mica decoder on one B200 (include/laya_decoder.h), mirroring Qwen35Model (Mica/Models/Qwen35Model.cs)
    with WeightPrecision.Q8_0: construct, `load(weights)` by checkpoint names, `forward(sequences, labels)` — every
    sequence from an empty state, returning each sequence's final-normed last hidden row (Qwen35Sequence.Hidden) and
    the label logits (Logits → TokenTable.QuantizedLogits) — `logits(hidden, ids)`, `layer(i, hidden, seq_lens)`;
    and with states: `new_state()`, `forward_sequences([Qwen35Sequence])`, `forward_state(tokens, state)`,
    `read(tokens, state)`."""

    def __init__(self, desc: DecoderDesc, device: int = 0):
        self.desc = desc
        h = ctypes.c_void_p()
        check(lib().laya_decoder_create(ctypes.byref(desc), device, ctypes.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().laya_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload(self, name: str, array: np.ndarray):
        a = np.ascontiguousarray(array)
        if a.dtype == np.float16:
            dt = F16
        else:
            a = np.ascontiguousarray(a, dtype=np.float32)
            dt = F32
        shape = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
        check(lib().laya_decoder_upload(self.handle, name.encode(), dt, shape, a.ndim, _np_ptr(a)))

    def upload_bf16_bits(self, name: str, bits: np.ndarray):
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        shape = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
        check(lib().laya_decoder_upload(self.handle, name.encode(), BF16, shape, a.ndim, _np_ptr(a)))

    def upload_q8_0(self, name: str, q: np.ndarray, d_fp16: np.ndarray):
        q = np.ascontiguousarray(q, dtype=np.int8)
        d = np.ascontiguousarray(d_fp16, dtype=np.float16).view(np.uint16)
        N, K = q.shape
        check(lib().laya_decoder_upload_q8_0(self.handle, name.encode(), _np_ptr(q), _np_ptr(d), N, K))

    def load(self, weights: Dict[str, np.ndarray]):
        for name, w in weights.items():
            if name.endswith("lm_head.weight"):
                continue
            self.upload(name, w)

    def missing(self) -> List[str]:
        n = ctypes.c_int()
        buf = ctypes.create_string_buffer(1 << 16)
        check(lib().laya_decoder_missing(self.handle, buf, len(buf), ctypes.byref(n)))
        return [x for x in buf.value.decode().split("\n") if x]

    @staticmethod
    def pack(sequences: Sequence[np.ndarray]):
        lens = _i32([len(s) for s in sequences])
        ids = _i32(np.concatenate([np.asarray(s, np.int64) for s in sequences]) if len(sequences) else [])
        return ids, lens

    def forward(self, sequences: Sequence[np.ndarray], labels: Optional[Sequence[int]] = None):
        """Returns (hidden [n_seq, hidden], logits [n_seq, n_labels] or None)."""
        ids, lens = self.pack(sequences)
        lab = None if labels is None else _i32(labels)
        hidden = np.zeros((len(sequences), self.desc.hidden), np.float32)
        logits = None if lab is None else np.zeros((len(sequences), len(lab)), np.float32)
        check(lib().laya_decoder_forward(self.handle, _np_ptr(ids), _np_ptr(lens), len(sequences), _np_ptr(lab),
                                         0 if lab is None else len(lab), _np_ptr(hidden), _np_ptr(logits)))
        return hidden, logits

    def new_state(self, capacity: int = 0) -> Qwen35State:
        """NewState (Qwen35Model.cs:419)."""
        h = ctypes.c_void_p()
        check(lib().laya_decoder_state_create(self.handle, capacity, ctypes.byref(h)))
        return Qwen35State(h)

    def forward_sequences(self, sequences: Sequence[Qwen35Sequence], labels: Optional[Sequence[int]] = None):
        """Forward(IReadOnlyList<Qwen35Sequence>) (Qwen35Model.cs:462-532): each sequence continues its state."""
        ids, lens = self.pack([q.tokens for q in sequences])
        n = len(sequences)
        states = (ctypes.c_void_p * max(1, n))(*[q.state.handle for q in sequences])
        readout = _i32([1 if q.readout else 0 for q in sequences])
        ncp = _i32([len(q.checkpoints) for q in sequences])
        cps = _i32([c for q in sequences for c in q.checkpoints])
        n_snap = int(ncp.sum())
        snaps = (ctypes.c_void_p * max(1, n_snap))()
        lab = None if labels is None else _i32(labels)
        hidden = np.zeros((n, self.desc.hidden), np.float32)
        logits = None if lab is None else np.zeros((n, len(lab)), np.float32)
        check(lib().laya_decoder_forward_states(self.handle, _np_ptr(ids), _np_ptr(lens), n, states, _np_ptr(readout),
                                                _np_ptr(ncp), _np_ptr(cps) if n_snap else None, snaps,
                                                _np_ptr(lab), 0 if lab is None else len(lab), _np_ptr(hidden),
                                                _np_ptr(logits)))
        k = 0
        for i, q in enumerate(sequences):
            q.hidden = hidden[i].copy() if q.readout else None
            q.logits = None if logits is None or not q.readout else logits[i].copy()
            q.snapshots = [Qwen35State(ctypes.c_void_p(snaps[k + j])) for j in range(len(q.checkpoints))]
            k += len(q.checkpoints)
        return sequences

    def forward_state(self, tokens, state: Qwen35State, labels: Optional[Sequence[int]] = None):
        """Forward(ReadOnlySpan<int>, Qwen35State) (Qwen35Model.cs:423-430): the final-normed hidden row of the last
        token (and the label logits when labels are given)."""
        q = self.forward_sequences([Qwen35Sequence(tokens, state)], labels)[0]
        return q.hidden if labels is None else (q.hidden, q.logits)

    def read(self, tokens, state: Qwen35State, checkpoints: Optional[Sequence[int]] = None):
        """Read (Qwen35Model.cs:436-439): tokens into the state without output; returns the checkpoint snapshots."""
        q = self.forward_sequences([Qwen35Sequence(tokens, state, readout=False, checkpoints=checkpoints)])[0]
        return q.snapshots

    def forward_device(self, ids_ptr: int, seq_lens: Sequence[int], labels: Sequence[int], hidden_ptr: int,
                       logits_ptr: int):
        lens, lab = _i32(seq_lens), _i32(labels)
        check(lib().laya_decoder_forward_device(self.handle, ctypes.c_void_p(ids_ptr), _np_ptr(lens), len(lens),
                                                _np_ptr(lab), len(lab), ctypes.c_void_p(hidden_ptr or 0),
                                                ctypes.c_void_p(logits_ptr or 0)))

    def logits(self, hidden: np.ndarray, ids: Sequence[int]) -> np.ndarray:
        h = _f32(hidden).reshape(-1, self.desc.hidden)
        lab = _i32(ids)
        out = np.zeros((h.shape[0], len(lab)), np.float32)
        check(lib().laya_decoder_logits(self.handle, _np_ptr(h), h.shape[0], _np_ptr(lab), len(lab), _np_ptr(out)))
        return out

    def layer(self, i: int, hidden: np.ndarray, seq_lens: Sequence[int]):
        """One layer on hidden [T, hidden]: returns (mixer output, layer output)."""
        x = _f32(hidden).copy()
        lens = _i32(seq_lens)
        mixer = np.zeros_like(x)
        check(lib().laya_decoder_layer(self.handle, i, _np_ptr(x), _np_ptr(lens), len(lens), _np_ptr(mixer)))
        return mixer, x

    def set_chunked_delta_rule(self, enabled: bool):
        """Stateless reads: the delta rule in 64-token tensor-core chunks (True) or the per-token sweep, bit-identical
        to the reference's (False, the default).  Reads through states always take the per-token sweep."""
        check(lib().laya_decoder_set_chunked_delta_rule(self.handle, 1 if enabled else 0))

    def record(self, enabled: bool):
        check(lib().laya_decoder_record_enable(self.handle, 1 if enabled else 0))

    def recorded(self, name: str, shape) -> np.ndarray:
        out = np.zeros(shape, np.float32)
        check(lib().laya_decoder_record_get(self.handle, name.encode(), _np_ptr(out), out.size))
        return out

    def synchronize(self):
        check(lib().laya_decoder_synchronize(self.handle))

    def set_stream(self, stream_handle: Optional[int]):
        check(lib().laya_decoder_set_stream(self.handle, ctypes.c_void_p(stream_handle or 0)))

    def launches(self) -> int:
        n = ctypes.c_longlong()
        check(lib().laya_decoder_launches(self.handle, ctypes.byref(n)))
        return n.value

    def set_profiling(self, enabled: bool):
        check(lib().laya_decoder_set_profiling(self.handle, 1 if enabled else 0))

    def profile(self, kind: int) -> Tuple[float, float, int]:
        ms, ops, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_longlong()
        check(lib().laya_decoder_profile(self.handle, kind, ctypes.byref(ms), ctypes.byref(ops), ctypes.byref(n)))
        return ms.value, ops.value, n.value
