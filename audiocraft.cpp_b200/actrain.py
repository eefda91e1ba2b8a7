"""ctypes binding of libactrain.so (include/actrain.h).

A thin mirror of the C ABI for Python callers (the tests and bench.py).  It mirrors the
reference trainer classes' vocabulary: `mf_step` is MfTrainGraph::compute plus
TrainAccumulation::add (src/mf/train.h:148-188), `optimizer` is TrainAccumulation::update
(src/ac/train_controls.h:89-118).  There is no CPU path: if the library cannot be loaded
every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libactrain.so")

ACT_OK, ACT_ERR_INVALID, ACT_ERR_CUDA, ACT_ERR_NCCL, ACT_ERR_STATE, ACT_ERR_NONFINITE = range(6)
FAMILY_MELODYFLOW, FAMILY_MUSICGEN = 0, 1
ADAPTER_LORA, ADAPTER_DORA_ROWS = 0, 1
TYPE_F32, TYPE_F16, TYPE_Q8_0 = 0, 1, 8
TARGETS = ("self.qkv", "self.out", "cross.q", "cross.kv", "cross.out", "ff.0", "ff.2")
# kernel families counted by act_path_counts (ACT_PATH_*)
PATHS = ("attn_fwd_tc", "attn_fwd_mma", "attn_bwd_tc", "attn_bwd_mma", "gemm_tc", "gemm_mma", "rank_tc",
         "rank_mma", "xattn_fwd_tc", "xattn_bwd_tc")


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("family", "dim", "layers", "heads", "head_dim", "ff_dim",
                                        "latent_dim", "cond_dim", "time_dim", "n_skip",
                                        "add_zero_attn", "n_q", "card", "special_token_id",
                                        "pos_denominator")] + \
               [("max_period", C.c_float), ("norm_eps", C.c_float)]


class AdapterDesc(C.Structure):
    _fields_ = [("type", C.c_int), ("rank", C.c_int), ("alpha", C.c_float),
                ("first_layer", C.c_int), ("targets", C.c_uint), ("seed", C.c_uint32),
                ("max_batch", C.c_int), ("frames", C.c_int), ("tokens", C.c_int),
                ("prefix_frames", C.c_int)]


class MfBatch(C.Structure):
    _fields_ = [("n", C.c_int), ("clean", C.c_void_p), ("noise", C.c_void_p),
                ("hidden", C.c_void_p), ("t", C.c_void_p), ("unconditional", C.c_void_p),
                ("valid_tokens", C.c_void_p), ("pivot", C.c_void_p), ("edit_start", C.c_void_p),
                ("stddev", C.c_void_p), ("sample_seed", C.c_uint64), ("window0", C.c_uint64)]


class MgBatch(C.Structure):
    _fields_ = [("n", C.c_int), ("codes", C.c_void_p), ("context", C.c_void_p)]


class Opt(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float), ("clip", C.c_float), ("step", C.c_int),
                ("count", C.c_int)]


class ActError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None

SIGNATURES = {
    "act_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.POINTER(ModelDesc), C.POINTER(AdapterDesc)]),
    "act_bind_weight": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t]),
    "act_finalize": (C.c_int, [C.c_void_p]),
    "act_param_count": (C.c_int64, [C.c_void_p]),
    "act_param_tensor_count": (C.c_int, [C.c_void_p]),
    "act_param_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_int64),
                                   C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "act_set_params": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "act_get_params": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "act_set_moments": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "act_get_grads": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "act_zero_grads": (C.c_int, [C.c_void_p]),
    "act_mf_step": (C.c_int, [C.c_void_p, C.POINTER(MfBatch), C.c_void_p]),
    "act_mg_step": (C.c_int, [C.c_void_p, C.POINTER(MgBatch), C.c_void_p]),
    "act_nccl_get_unique_id": (C.c_int, [C.c_void_p]),
    "act_nccl_init": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "act_allreduce_grads": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "act_set_grad_sync": (C.c_int, [C.c_void_p, C.c_int]),
    "act_set_timeout": (C.c_int, [C.c_void_p, C.c_int64]),
    "act_optimizer": (C.c_int, [C.c_void_p, C.POINTER(Opt), C.POINTER(C.c_int)]),
    "act_last_error": (C.c_char_p, [C.c_void_p]),
    "act_destroy": (None, [C.c_void_p]),
    "act_stream": (C.c_void_p, [C.c_void_p]),
    "act_mf_stage": (C.c_int, [C.c_void_p, C.POINTER(MfBatch)]),
    "act_mg_stage": (C.c_int, [C.c_void_p, C.POINTER(MgBatch)]),
    "act_run_staged": (C.c_int, [C.c_void_p, C.c_void_p]),
    "act_set_profiling": (C.c_int, [C.c_void_p, C.c_int]),
    "act_kernel_stats": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                   C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "act_reset_kernel_stats": (C.c_int, [C.c_void_p]),
    "act_step_flops": (C.c_double, [C.c_void_p, C.c_int]),
    "act_graph_kernel_nodes": (C.c_int64, [C.c_void_p, C.c_int]),
    "act_attention": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "act_attention_bwd_noalloc": (C.c_int, [C.c_void_p] * 6 + [C.c_void_p] * 3 + [C.c_int] * 4 +
                                  [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "act_gemm_f16": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "act_gemm_q8_0": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "act_gelu_f16": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int]),
    "act_path_counts": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.c_int]),
    "act_wait_probe": (C.c_int, [C.c_void_p, C.c_int64]),
    "act_mg_staged": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]),
    "act_q8_0_dequant": (C.c_int, [C.c_int, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "act_set_deterministic": (C.c_int, [C.c_void_p, C.c_int]),
    "act_mf_staged": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "act_lora_linear": (C.c_int, [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                  C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_float, C.c_void_p]),
    "act_rank_gemm_f16": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "act_rank_gemm_q8_0": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.POINTER(C.c_float)]),
}


def lib():
    """Load libactrain.so; raises if it is missing (there is no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ActError(ACT_ERR_STATE, f"{LIB_PATH} is not built: run audiocraft.cpp_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


class Context:
    """One device context: MfTrainGraph / MgTrainGraph equivalent for a batch of samples."""

    def __init__(self, model: ModelDesc, adapter: AdapterDesc, device: int = 0):
        self._L = lib()
        self.model, self.adapter = model, adapter
        h = C.c_void_p()
        rc = self._L.act_create(C.byref(h), device, C.byref(model), C.byref(adapter))
        if rc != ACT_OK:
            raise ActError(rc, self._L.act_last_error(None).decode())
        self.h = h
        self._keep = []

    def _check(self, rc):
        if rc != ACT_OK:
            raise ActError(rc, self._L.act_last_error(self.h).decode())

    def close(self):
        if getattr(self, "h", None):
            self._L.act_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ----------------------------------------------------------------- weights
    def bind(self, name: str, array: np.ndarray, ggml_type: int = TYPE_F32):
        a = np.ascontiguousarray(array)
        self._check(self._L.act_bind_weight(self.h, name.encode(), ggml_type, a.ctypes.data, a.nbytes))

    def finalize(self):
        self._check(self._L.act_finalize(self.h))
        self.n = int(self._L.act_param_count(self.h))

    # ----------------------------------------------------------------- parameters
    def param_table(self):
        out = []
        buf = C.create_string_buffer(256)
        for i in range(self._L.act_param_tensor_count(self.h)):
            off, r, c = C.c_int64(), C.c_int64(), C.c_int64()
            self._check(self._L.act_param_tensor(self.h, i, buf, 256, C.byref(off), C.byref(r), C.byref(c)))
            out.append((buf.value.decode(), off.value, (r.value, c.value)))
        return out

    def get_params(self):
        v, m, s = (np.zeros(self.n, np.float32) for _ in range(3))
        self._check(self._L.act_get_params(self.h, v.ctypes.data, m.ctypes.data, s.ctypes.data, self.n))
        return v, m, s

    def set_params(self, v):
        v = np.ascontiguousarray(v, np.float32)
        self._check(self._L.act_set_params(self.h, v.ctypes.data, v.size))

    def set_moments(self, m, v):
        m = np.ascontiguousarray(m, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self._check(self._L.act_set_moments(self.h, m.ctypes.data, v.ctypes.data, m.size))

    def get_grads(self):
        g = np.zeros(self.n, np.float32)
        self._check(self._L.act_get_grads(self.h, g.ctypes.data, self.n))
        return g

    def zero_grads(self):
        self._check(self._L.act_zero_grads(self.h))

    # ----------------------------------------------------------------- steps
    def _mf_batch(self, clean, noise, hidden, t, unconditional=None, valid_tokens=None, pivot=None,
                  edit_start=None, stddev=None, sample_seed=0, window0=0):
        f32 = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)
        arrs = [f32(clean), f32(noise), f32(hidden), f32(t),
                None if unconditional is None else np.ascontiguousarray(unconditional, np.int32),
                None if valid_tokens is None else np.ascontiguousarray(valid_tokens, np.int32),
                f32(pivot), f32(edit_start), f32(stddev)]
        self._keep = arrs
        return MfBatch(arrs[0].shape[0], *[_ptr(a) for a in arrs], sample_seed, window0)

    def mf_step(self, clean, noise, hidden, t, unconditional=None, valid_tokens=None, pivot=None,
                edit_start=None, stddev=None, sample_seed=0, window0=0):
        """One microbatch; with pivot/edit_start the edit-bridge objective (noise unused); with stddev
        the device draws clean = clean + stddev * z and the noise itself (noise unused)."""
        b = self._mf_batch(clean, noise, hidden, t, unconditional, valid_tokens, pivot, edit_start, stddev,
                           sample_seed, window0)
        loss = np.zeros(b.n, np.float32)
        self._check(self._L.act_mf_step(self.h, C.byref(b), loss.ctypes.data))
        return loss

    def mf_stage(self, clean, noise, hidden, t, unconditional=None, valid_tokens=None):
        b = self._mf_batch(clean, noise, hidden, t, unconditional, valid_tokens)
        self._check(self._L.act_mf_stage(self.h, C.byref(b)))
        return b.n

    def set_deterministic(self, on: bool = True):
        """act_set_deterministic: bit-for-bit reproducible steps (ordered dQ adds)."""
        self._check(self._L.act_set_deterministic(self.h, int(on)))

    def mf_staged(self, n, lat, T):
        """The clean / noise windows the device holds for the last MelodyFlow batch."""
        c = np.zeros((n, lat, T), np.float32)
        z = np.zeros((n, lat, T), np.float32)
        self._check(self._L.act_mf_staged(self.h, c.ctypes.data, z.ctypes.data, c.size))
        return c, z

    def mg_step(self, codes, context):
        arrs = [np.ascontiguousarray(codes, np.int32), np.ascontiguousarray(context, np.float32)]
        self._keep = arrs
        b = MgBatch(arrs[0].shape[0], arrs[0].ctypes.data, arrs[1].ctypes.data)
        loss = np.zeros(b.n, np.float32)
        self._check(self._L.act_mg_step(self.h, C.byref(b), loss.ctypes.data))
        return loss

    def mg_stage(self, codes, context):
        arrs = [np.ascontiguousarray(codes, np.int32), np.ascontiguousarray(context, np.float32)]
        self._keep = arrs
        b = MgBatch(arrs[0].shape[0], arrs[0].ctypes.data, arrs[1].ctypes.data)
        self._check(self._L.act_mg_stage(self.h, C.byref(b)))
        return b.n

    def run_staged(self, n=None, read_loss=True):
        if read_loss:
            loss = np.zeros(n, np.float32)
            self._check(self._L.act_run_staged(self.h, loss.ctypes.data))
            return loss
        self._check(self._L.act_run_staged(self.h, None))
        return None

    def optimizer(self, lr, step, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, clip=1.0, count=0):
        o = Opt(lr, beta1, beta2, eps, weight_decay, clip, step, count)
        bad = C.c_int(0)
        rc = self._L.act_optimizer(self.h, C.byref(o), C.byref(bad))
        if rc != ACT_OK:
            raise ActError(rc, self._L.act_last_error(self.h).decode())
        return bad.value

    # ----------------------------------------------------------------- data parallel
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        rc = lib().act_nccl_get_unique_id(buf)
        if rc != ACT_OK:
            raise ActError(rc, lib().act_last_error(None).decode())
        return buf.raw

    def nccl_init(self, uid: bytes, nranks: int, rank: int):
        buf = C.create_string_buffer(uid, 128)
        self._check(self._L.act_nccl_init(self.h, buf, nranks, rank))

    def allreduce_grads(self, global_count: int):
        self._check(self._L.act_allreduce_grads(self.h, None, global_count))

    def set_grad_sync(self, global_count: int):
        """act_set_grad_sync: the next step all-reduces its gradients in-step (per-layer buckets)."""
        self._check(self._L.act_set_grad_sync(self.h, global_count))

    def set_timeout(self, ms: int):
        """act_set_timeout: bound on NCCL initialisation and on host waits while a communicator lives."""
        self._check(self._L.act_set_timeout(self.h, int(ms)))

    # ----------------------------------------------------------------- measurement
    def stream(self) -> int:
        return self._L.act_stream(self.h)

    def set_profiling(self, on: bool):
        self._check(self._L.act_set_profiling(self.h, int(on)))

    def kernel_stats(self, cls: int):
        ms, fl, by, n = C.c_double(), C.c_double(), C.c_double(), C.c_int64()
        self._check(self._L.act_kernel_stats(self.h, cls, C.byref(ms), C.byref(fl), C.byref(by), C.byref(n)))
        return {"ms": ms.value, "flops": fl.value, "bytes": by.value, "launches": n.value}

    def reset_kernel_stats(self):
        self._check(self._L.act_reset_kernel_stats(self.h))

    def step_flops(self, n: int) -> float:
        return float(self._L.act_step_flops(self.h, n))

    def graph_kernel_nodes(self, n: int) -> int:
        return int(self._L.act_graph_kernel_nodes(self.h, n))

    def path_counts(self) -> dict:
        """Launches issued so far per kernel family (act_path_counts)."""
        buf = (C.c_int64 * len(PATHS))()
        self._check(self._L.act_path_counts(self.h, buf, len(PATHS)))
        return dict(zip(PATHS, list(buf)))

    def wait_probe(self, limit_ns: int):
        """act_wait_probe: a bounded device wait on a flag nothing sets; raises ActError."""
        self._check(self._L.act_wait_probe(self.h, int(limit_ns)))

    def mg_staged(self, n: int, n_q: int, steps: int, selected: int):
        """Staged delayed ids [n][n_q][steps] and targets [n][n_q][selected] (act_mg_staged)."""
        ids = np.zeros((n, n_q, steps), np.int32)
        tgt = np.zeros((n, n_q, selected), np.int32)
        self._check(self._L.act_mg_staged(self.h, ids.ctypes.data, ids.size, tgt.ctypes.data, tgt.size))
        return ids, tgt


def gemm_f16(A_bits: np.ndarray, B_bits: np.ndarray, M: int, N: int, K: int, b_mn_major: bool, path: int = 0,
              device: int = 0, reps: int = 0):
    """C = A . B(n,k) on the device; A_bits/B_bits are f16 bit patterns (uint16).  With reps > 0
    returns (C, mean ms per call)."""
    C_ = np.zeros((M, N), np.float32)
    a = np.ascontiguousarray(A_bits, np.uint16)
    b = np.ascontiguousarray(B_bits, np.uint16)
    ms = C.c_float(0.0)
    rc = lib().act_gemm_f16(device, a.ctypes.data, b.ctypes.data, C_.ctypes.data, M, N, K, int(b_mn_major), path,
                             reps, C.byref(ms))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return (C_, ms.value) if reps > 0 else C_


def gemm_q8_0(A_bits: np.ndarray, B_blocks: np.ndarray, M: int, N: int, K: int, b_mn_major: bool, path: int = 0,
              device: int = 0, reps: int = 0):
    """C = A . B(n,k) with B as the Q8_0 blocks of the weight ([N][K], or [K][N] when b_mn_major),
    dequantised inside the GEMM.  With reps > 0 returns (C, mean ms per call)."""
    C_ = np.zeros((M, N), np.float32)
    a = np.ascontiguousarray(A_bits, np.uint16)
    b = np.ascontiguousarray(B_blocks, np.uint8)
    ms = C.c_float(0.0)
    rc = lib().act_gemm_q8_0(device, a.ctypes.data, b.ctypes.data, C_.ctypes.data, M, N, K, int(b_mn_major), path,
                             reps, C.byref(ms))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return (C_, ms.value) if reps > 0 else C_


def gelu_f16(z_bits: np.ndarray, direct: bool, device: int = 0):
    """act_gelu_f16: (gelu bits, gelu' bits) of f16 inputs, element by element (direct) or by the
    training step's vectorised pass."""
    z = np.ascontiguousarray(z_bits, np.uint16)
    g = np.zeros_like(z)
    dg = np.zeros_like(z)
    rc = lib().act_gelu_f16(device, z.ctypes.data, g.ctypes.data, dg.ctypes.data, z.size, int(direct))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return g, dg


def q8_0_dequant(blocks: np.ndarray, device: int = 0):
    """act_q8_0_dequant: (fp32 d*q, its f16 bit patterns) of Q8_0 blocks ([nblocks][34] bytes)."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1)
    nb = b.size // 34
    f = np.zeros(nb * 32, np.float32)
    h = np.zeros(nb * 32, np.uint16)
    rc = lib().act_q8_0_dequant(device, b.ctypes.data, nb, f.ctypes.data, h.ctypes.data)
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return f, h


def lora_linear(x: np.ndarray, w: np.ndarray, w_type: int, out: int, A=None, B=None, alpha: float = 1.0,
                magnitude=None, strength: float = 1.0, device: int = 0) -> np.ndarray:
    """act_lora_linear: y = W x with a LoRA / DoRA-rows adapter applied (inference, src/ac/lora.h:50-83).
    x [rows][in] fp32; w the weight's raw data (fp32 values, f16 bit patterns or Q8_0 blocks)."""
    xa = np.ascontiguousarray(x, np.float32)
    rows, n_in = xa.shape
    wa = np.ascontiguousarray(w)
    keep = [xa, wa]
    ptr = lambda a: None if a is None else keep.append(np.ascontiguousarray(a, np.float32)) or keep[-1].ctypes.data
    pa, pb, pm = ptr(A), ptr(B), ptr(magnitude)
    rank = 0 if A is None else np.asarray(A).shape[0]
    y = np.zeros((rows, out), np.float32)
    rc = lib().act_lora_linear(device, xa.ctypes.data, rows, n_in, out, w_type, wa.ctypes.data, wa.nbytes, pa, pb, rank,
                               alpha, pm, strength, y.ctypes.data)
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return y


RANK_ACC, RANK_ACC_T, RANK_STORE = 0, 1, 2


def rank_gemm_f16(A_bits: np.ndarray, B_bits: np.ndarray, M: int, K: int, nb: int, a_mn: bool, b_mn: bool,
                   kind: int, alpha: float = 1.0, C_init: np.ndarray | None = None, splits: int = 0, device: int = 0,
                   reps: int = 0):
    """Rank-block product C = alpha A(M x K) B(K x nb) (act_rank_gemm_f16).  A_bits is [M][K]
    (a_mn False) or [K][M]; B_bits is [nb][K] (b_mn False) or [K][nb].  kind RANK_ACC returns
    C_init + C ([M][nb]), RANK_ACC_T returns C_init + C^T ([nb][M]), RANK_STORE returns f16(C).
    With reps > 0 returns (C, mean ms per call)."""
    shape = (nb, M) if kind == RANK_ACC_T else (M, nb)
    C_ = np.zeros(shape, np.float32) if C_init is None else np.ascontiguousarray(C_init, np.float32).copy()
    a = np.ascontiguousarray(A_bits, np.uint16)
    b = np.ascontiguousarray(B_bits, np.uint16)
    ms = C.c_float(0.0)
    rc = lib().act_rank_gemm_f16(device, kind, a.ctypes.data, b.ctypes.data, C_.ctypes.data, M, K, nb, int(a_mn),
                                  int(b_mn), float(alpha), splits, reps, C.byref(ms))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return (C_, ms.value) if reps > 0 else C_



def rank_gemm_q8_0(W_blocks: np.ndarray, B_bits: np.ndarray, M: int, K: int, nb: int, a_mn: bool, b_mn: bool,
                   kind: int, alpha: float = 1.0, C_init: np.ndarray | None = None, splits: int = 0, device: int = 0,
                   reps: int = 0):
    """act_rank_gemm_q8_0: rank_gemm_f16 with A read from a weight given as its Q8_0 blocks
    ([M][K] when a_mn is False, [K][M] when True), kept quantised on the device."""
    shape = (nb, M) if kind == RANK_ACC_T else (M, nb)
    C_ = np.zeros(shape, np.float32) if C_init is None else np.ascontiguousarray(C_init, np.float32).copy()
    w = np.ascontiguousarray(W_blocks, np.uint8)
    b = np.ascontiguousarray(B_bits, np.uint16)
    ms = C.c_float(0.0)
    rc = lib().act_rank_gemm_q8_0(device, kind, w.ctypes.data, b.ctypes.data, C_.ctypes.data, M, K, nb, int(a_mn),
                                   int(b_mn), float(alpha), splits, reps, C.byref(ms))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return (C_, ms.value) if reps > 0 else C_

def attention(q, k, v, dout, clips, T, Tk, H, nvalid=None, causal=False, zero_key=False, rope=None, device=0):
    """Kernel-level attention: f16 bit-pattern inputs (uint16) -> dict of outputs and device times."""
    D = H * 64
    o = np.zeros((clips * T, D), np.uint16)
    lse = np.zeros((clips, H, T), np.float32)
    dq = np.zeros((clips * T, D), np.uint16)
    dk = np.zeros((clips * Tk, D), np.uint16)
    dv = np.zeros((clips * Tk, D), np.uint16)
    arrs = [np.ascontiguousarray(x, np.uint16) for x in (q, k, v)]
    d = None if dout is None else np.ascontiguousarray(dout, np.uint16)
    nv = None if nvalid is None else np.ascontiguousarray(nvalid, np.int32)
    rp = None if rope is None else np.ascontiguousarray(rope, np.float32)
    mf, mb = C.c_float(), C.c_float()
    rc = lib().act_attention(device, arrs[0].ctypes.data, arrs[1].ctypes.data, arrs[2].ctypes.data, _ptr(d), clips, T,
                             Tk, H, _ptr(nv), int(causal), int(zero_key), _ptr(rp), o.ctypes.data, lse.ctypes.data,
                             dq.ctypes.data if d is not None else None, dk.ctypes.data if d is not None else None,
                             dv.ctypes.data if d is not None else None, C.byref(mf), C.byref(mb))
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())
    return {"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv, "ms_fwd": mf.value, "ms_bwd": mb.value}


NOALLOC_ATTN_SCRATCH_FLOATS = 8 * 1024 * 1024


def attention_bwd_noalloc(q, k, v, o, lse, dout, dq, dk, dv, clips, T, Tk, H, nvalid=0, causal=False,
                          zero_key=False, rope=0, stream=0):
    """act_attention_bwd_noalloc: every argument is a device address (int), including the outputs."""
    rc = lib().act_attention_bwd_noalloc(q, k, v, o, lse, dout, dq, dk, dv, clips, T, Tk, H, nvalid or None,
                                         int(causal), int(zero_key), rope or None, stream or None)
    if rc != ACT_OK:
        raise ActError(rc, lib().act_last_error(None).decode())


def mf_model(dim, layers, heads, ff_dim, latent_dim=128, cond_dim=768, time_dim=256, norm_eps=1e-5):
    return ModelDesc(FAMILY_MELODYFLOW, dim, layers, heads, dim // heads, ff_dim, latent_dim, cond_dim,
                     time_dim, (layers - 1) // 2, 1, 0, 0, 0, 0, 10000.0, norm_eps)


def mg_model(dim, layers, heads, ff_dim, n_q=4, card=2048, norm_eps=1e-5, max_period=10000.0):
    return ModelDesc(FAMILY_MUSICGEN, dim, layers, heads, dim // heads, ff_dim, 0, 0, 0, 0, 0, n_q, card,
                     card, dim // 2 - 1, max_period, norm_eps)
