"""ctypes binding of libspo_cuda.so (the C ABI declared in include/spo_cuda.h).

The library is loaded from this package directory; there is no fallback of any
kind: if the shared object is missing, importing the binding raises. Every call's
int status is checked and a nonzero status raises SpoError with the library's own
message (spo_last_error_string).

Pointers are passed as integers (``tensor.data_ptr()``) and streams as the raw
cudaStream_t handle (``torch.cuda.Stream.cuda_stream``).
"""

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libspo_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "spo_cuda.h")

MAX_LAYERS = 8
NUM_STATS = 8
REPORT_SIZE = 16
COMM_ID_BYTES = 128
ALIGN_FLOATS = 64

STAT = {"actor_loss": 0, "ce": 1, "entropy": 2, "kl_q": 3, "kl_old": 4, "critic_loss": 5}
REPORT = {"norm_actor": 0, "norm_critic": 1, "clip_actor": 4, "clip_critic": 5,
          "dlog_alpha": 8, "step": 9}

ERRORS = {0: "SPO_OK", -1: "SPO_ERR_ARG", -2: "SPO_ERR_SHAPE", -3: "SPO_ERR_ALIGN",
          -4: "SPO_ERR_WORKSPACE", -5: "SPO_ERR_CUDA", -6: "SPO_ERR_NCCL",
          -7: "SPO_ERR_UNSUPPORTED", -8: "SPO_ERR_TIMEOUT"}


class SpoError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class MlpDesc(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("dims", ctypes.c_int32 * (MAX_LAYERS + 1))]

    @classmethod
    def of(cls, dims):
        d = cls()
        if dims is None:
            d.num_layers = 0
            return d
        d.num_layers = len(dims) - 1
        for i, v in enumerate(dims):
            d.dims[i] = int(v)
        return d


class TcGemmDesc(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("a_hi", ctypes.c_void_p), ("a_lo", ctypes.c_void_p),
                ("b_hi", ctypes.c_void_p), ("b_lo", ctypes.c_void_p), ("m", ctypes.c_int64),
                ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("k_chunk", ctypes.c_int64),
                ("bias", ctypes.c_void_p), ("mask", ctypes.c_void_p), ("c_hi", ctypes.c_void_p),
                ("c_lo", ctypes.c_void_p), ("c_part", ctypes.c_void_p), ("colsum", ctypes.c_void_p),
                ("err", ctypes.c_void_p), ("mask_bits", ctypes.c_void_p), ("c_bits", ctypes.c_void_p)]


TC_FWD, TC_DX, TC_DX_F32, TC_DW = 0, 1, 2, 3


class LearnerDesc(ctypes.Structure):
    _fields_ = [("actor", MlpDesc), ("critic", MlpDesc), ("max_rows", ctypes.c_int64),
                ("lr_actor", ctypes.c_float), ("lr_critic", ctypes.c_float),
                ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("adam_eps", ctypes.c_float),
                ("max_grad_norm", ctypes.c_float), ("kl_eps", ctypes.c_float),
                ("use_kl", ctypes.c_int32), ("dual", ctypes.c_int32), ("engine", ctypes.c_int32)]


class LearnerLayout(ctypes.Structure):
    _fields_ = [("actor_offset", ctypes.c_int64), ("actor_size", ctypes.c_int64),
                ("critic_offset", ctypes.c_int64), ("critic_size", ctypes.c_int64),
                ("alpha_index", ctypes.c_int64), ("stats_offset", ctypes.c_int64),
                ("total", ctypes.c_int64),
                ("actor_w_off", ctypes.c_int64 * MAX_LAYERS), ("actor_b_off", ctypes.c_int64 * MAX_LAYERS),
                ("critic_w_off", ctypes.c_int64 * MAX_LAYERS), ("critic_b_off", ctypes.c_int64 * MAX_LAYERS)]


class Batch(ctypes.Structure):
    _fields_ = [("obs", ctypes.c_void_p), ("mask", ctypes.c_void_p), ("q", ctypes.c_void_p),
                ("logits_old", ctypes.c_void_p), ("target", ctypes.c_void_p),
                ("rows", ctypes.c_int64), ("cells", ctypes.c_void_p)]


class TrainState(ctypes.Structure):
    _fields_ = [("params", ctypes.c_void_p), ("grads", ctypes.c_void_p),
                ("adam_m", ctypes.c_void_p), ("adam_v", ctypes.c_void_p),
                ("step", ctypes.c_void_p), ("report", ctypes.c_void_p)]


P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
F = ctypes.c_float
SZ = ctypes.c_size_t
INT = ctypes.c_int

# name: (restype, [argtypes]); status-returning functions have restype INT
SIGNATURES = {
    "spo_abi_version": (I32, []),
    "spo_last_error_string": (ctypes.c_char_p, []),
    "spo_linear_fwd": (INT, [P, P, P, P, P, I64, I64, I64, I32]),
    "spo_linear_bwd_workspace_size": (SZ, [I64, I64, I64]),
    "spo_linear_bwd": (INT, [P, P, P, P, P, P, P, P, I64, I64, I64, P, SZ]),
    "spo_linear_bwd_noalloc": (INT, [P, P, P, P, P, P, P, P, I64, I64, I64]),
    "spo_relu": (INT, [P, P, I64]),
    "spo_relu_bwd": (INT, [P, P, P, I64]),
    "spo_mlp_param_layout": (INT, [ctypes.POINTER(MlpDesc), ctypes.POINTER(I64), ctypes.POINTER(I64),
                                   ctypes.POINTER(I64)]),
    "spo_mlp_acts_size": (I64, [ctypes.POINTER(MlpDesc), I64]),
    "spo_mlp_fwd": (INT, [P, ctypes.POINTER(MlpDesc), P, P, I64, P, P]),
    "spo_mlp_bwd_workspace_size": (SZ, [ctypes.POINTER(MlpDesc), I64]),
    "spo_mlp_bwd": (INT, [P, ctypes.POINTER(MlpDesc), P, P, P, P, I64, P, P, SZ]),
    "spo_mask_logits": (INT, [P, P, P, I64]),
    "spo_softmax_rows": (INT, [P, P, P, I64, I32]),
    "spo_log_softmax_rows": (INT, [P, P, P, I64, I32]),
    "spo_logsumexp_rows": (INT, [P, P, P, I64, I32]),
    "spo_cross_entropy_rows": (INT, [P, P, P, P, I64, I32]),
    "spo_entropy_rows": (INT, [P, P, P, I64, I32]),
    "spo_kl_rows": (INT, [P, P, P, P, I64]),
    "spo_logits_grad": (INT, [P, P, P, P, P, I64, F]),
    "spo_value_loss_grad": (INT, [P, P, P, P, I64, F]),
    "spo_head_workspace_size": (SZ, [I64, I32, I32]),
    "spo_actor_head_fwd_bwd": (INT, [P, P, P, P, I64, I32, I32, P, P, P, P, F, P, P, P, P, P, P, P,
                                     P, P, SZ]),
    "spo_critic_head_fwd_bwd": (INT, [P, P, P, P, I64, I32, P, F, P, P, P, P, P, P, P, P, SZ]),
    "spo_loss_workspace_size": (SZ, []),
    "spo_actor_loss_fwd_bwd": (INT, [P, P, P, P, P, P, F, I64, I32, F, P, P, P, P, SZ]),
    "spo_value_loss_fwd_bwd": (INT, [P, P, P, I64, F, P, P, P, SZ]),
    "spo_sum_squares_workspace_size": (SZ, []),
    "spo_sum_squares": (INT, [P, P, I64, P, P, SZ]),
    "spo_global_clip_scale": (F, [F, F]),
    "spo_adam_flat": (INT, [P, P, P, P, P, I64, F, F, F, F, I32, F]),
    "spo_ema": (INT, [P, P, P, I64, F]),
    "spo_truncated_gae": (INT, [P, P, P, P, P, P, P, P, I64, I32, F]),
    "spo_measure_peaks": (INT, [P, P, P]),
    "spo_replay_sample": (INT, [P, P, I64, I64, ctypes.c_uint32, ctypes.c_uint32]),
    "spo_replay_gather": (INT, [P, P, P, P, I64, I64, I64, P]),
    "spo_encode_obs": (INT, [P, P, P, P, I64]),
    "spo_tc_gemm_shape": (INT, [ctypes.POINTER(TcGemmDesc), ctypes.POINTER(I32), ctypes.POINTER(I32)]),
    "spo_tc_gemm": (INT, [P, ctypes.POINTER(TcGemmDesc)]),
    "spo_tc_gemm_withheld": (INT, [P, ctypes.POINTER(TcGemmDesc), I64]),
    "spo_split_tf32": (INT, [P, P, P, P, I64, I32]),
    "spo_learner_layout_of": (INT, [ctypes.POINTER(LearnerDesc), ctypes.POINTER(LearnerLayout)]),
    "spo_learner_workspace_size": (SZ, [ctypes.POINTER(LearnerDesc)]),
    "spo_learner_create": (INT, [ctypes.POINTER(LearnerDesc), P, SZ, ctypes.POINTER(P)]),
    "spo_learner_destroy": (INT, [P]),
    "spo_learner_backward": (INT, [P, P, ctypes.POINTER(Batch), F, ctypes.POINTER(TrainState)]),
    "spo_learner_apply": (INT, [P, P, ctypes.POINTER(TrainState)]),
    "spo_learner_step": (INT, [P, P, ctypes.POINTER(Batch), ctypes.POINTER(TrainState)]),
    "spo_learner_set_small_rows": (INT, [P, I64]),
    "spo_learner_step_withheld": (INT, [P, P, ctypes.POINTER(Batch), ctypes.POINTER(TrainState), I64]),
    "spo_learner_status": (INT, [P, ctypes.POINTER(I32)]),
    "spo_learner_cache": (INT, [P, I32, I32, ctypes.POINTER(P), ctypes.POINTER(P)]),
    "spo_learner_forward": (INT, [P, P, I32, P, P, P, I64, P, P]),
    "spo_comm_get_unique_id": (INT, [P]),
    "spo_comm_init": (INT, [ctypes.POINTER(P), P, I32, I32]),
    "spo_comm_destroy": (INT, [P]),
    "spo_allreduce_sum": (INT, [P, P, P, I64]),
}

_lib = None


def header_symbols():
    """Function names declared in include/spo_cuda.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^SPO_API [\w\* ]+?\b(spo_\w+)\(", text, flags=re.M)))


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m spo_mojo_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    return lib().spo_last_error_string().decode(errors="replace")


def check(rc):
    if rc != 0:
        raise SpoError(rc, last_error())
    return rc


def call(name, *args):
    """Call a status-returning entry point and raise on failure."""
    return check(getattr(lib(), name)(*args))


def ptr(t):
    """Device (or host) address of a tensor, or None for a missing optional argument."""
    if t is None:
        return None
    return t.data_ptr()
