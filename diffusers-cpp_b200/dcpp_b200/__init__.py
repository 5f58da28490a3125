"""Python binding of libdcpp_b200.so, the B200 (sm_100a) Flux2 DiT denoise path.

Thin ctypes wrapper over the C ABI declared in ``include/dcpp.h``; all
arithmetic runs in the library's CUDA kernels.  There is no fallback: if the
shared library is missing, importing ``lib()`` raises.

The classes mirror the reference's C++ surface:
``Flux2Model`` <-> ``Flux2Transformer2DModel`` (config, parameter binding by
GGUF name, ``forward``) plus ``Flux2KleinPipeline::denoise``.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from typing import Iterable, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdcpp_b200.so")

DCPP_OK = 0
DCPP_ERR_INVALID_ARG = 1
STATUS_NAMES = {
    0: "DCPP_OK", 1: "DCPP_ERR_INVALID_ARG", 2: "DCPP_ERR_UNSUPPORTED", 3: "DCPP_ERR_CUDA",
    4: "DCPP_ERR_NCCL", 5: "DCPP_ERR_TIMEOUT", 6: "DCPP_ERR_OOM", 7: "DCPP_ERR_STATE",
    8: "DCPP_ERR_NOT_FOUND", 9: "DCPP_ERR_INJECTED",
}

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_BF16 = 0, 1, 8, 12, 30
NCCL_ID_BYTES = 128

_c_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p


class DcppError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Flux2ConfigC(ctypes.Structure):
    _fields_ = [
        ("patch_size", ctypes.c_int64),
        ("in_channels", ctypes.c_int64),
        ("out_channels", ctypes.c_int64),
        ("num_layers", ctypes.c_int64),
        ("num_single_layers", ctypes.c_int64),
        ("attention_head_dim", ctypes.c_int64),
        ("num_attention_heads", ctypes.c_int64),
        ("joint_attention_dim", ctypes.c_int64),
        ("timestep_guidance_channels", ctypes.c_int64),
        ("mlp_ratio", ctypes.c_float),
        ("n_axes", ctypes.c_int64),
        ("axes_dims_rope", ctypes.c_int64 * 8),
        ("rope_theta", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("guidance_embeds", ctypes.c_int32),
    ]


class FlowMatchConfigC(ctypes.Structure):
    """dcpp_flow_match_config (the scheduler's constructor options)."""
    _fields_ = [
        ("num_train_timesteps", ctypes.c_int32),
        ("shift", ctypes.c_float),
        ("use_dynamic_shifting", ctypes.c_int32),
        ("has_shift_terminal", ctypes.c_int32),
        ("shift_terminal", ctypes.c_float),
        ("invert_sigmas", ctypes.c_int32),
        ("time_shift_type", ctypes.c_int32),
    ]


class Qwen3ConfigC(ctypes.Structure):
    _fields_ = [
        ("vocab_size", ctypes.c_int64),
        ("hidden_size", ctypes.c_int64),
        ("intermediate_size", ctypes.c_int64),
        ("num_hidden_layers", ctypes.c_int64),
        ("num_attention_heads", ctypes.c_int64),
        ("num_key_value_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
    ]


class VAEConfigC(ctypes.Structure):
    _fields_ = [
        ("in_channels", ctypes.c_int64),
        ("out_channels", ctypes.c_int64),
        ("block_out_channels", ctypes.c_int64 * 8),
        ("n_blocks", ctypes.c_int32),
        ("layers_per_block", ctypes.c_int64),
        ("latent_channels", ctypes.c_int64),
        ("norm_num_groups", ctypes.c_int64),
        ("sample_size", ctypes.c_int64),
        ("force_upcast", ctypes.c_int32),
        ("use_quant_conv", ctypes.c_int32),
        ("use_post_quant_conv", ctypes.c_int32),
        ("mid_block_add_attention", ctypes.c_int32),
        ("batch_norm_eps", ctypes.c_float),
        ("batch_norm_momentum", ctypes.c_float),
        ("patch_size", ctypes.c_int64 * 2),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "dcpp_version": (ctypes.c_char_p, []),
    "dcpp_init": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_vp)]),
    "dcpp_destroy": (ctypes.c_int, [_vp]),
    "dcpp_last_error": (ctypes.c_char_p, [_vp]),
    "dcpp_set_stream": (ctypes.c_int, [_vp, _vp]),
    "dcpp_synchronize": (ctypes.c_int, [_vp]),
    "dcpp_alloc": (ctypes.c_int, [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]),
    "dcpp_free": (ctypes.c_int, [_vp, _vp]),
    "dcpp_memcpy": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_size_t]),
    "dcpp_row_bytes": (ctypes.c_int, [ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]),
    "dcpp_inject_fault": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int]),
    "dcpp_set_gemm_kernel": (ctypes.c_int, [_vp, ctypes.c_int]),
    "dcpp_set_attention_kernel": (ctypes.c_int, [_vp, ctypes.c_int]),
    "dcpp_set_wait_timeout": (ctypes.c_int, [_vp, ctypes.c_double]),
    "dcpp_tp_barrier_selftest": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_uint32]),
    "dcpp_dequant": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, _vp]),
    "dcpp_dequant_bf16": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, _vp]),
    "dcpp_f32_to_bf16": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, _vp]),
    "dcpp_gemm": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int64, _vp]),
    "dcpp_gemm_noalloc": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int64,
                                         _vp]),
    "dcpp_packed_bytes": (ctypes.c_int, [ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]),
    "dcpp_pack_weight": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp]),
    "dcpp_gemm_packed": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int64,
                                        _vp]),
    "dcpp_layernorm_mod": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp, _vp, ctypes.c_float, _vp]),
    "dcpp_attention": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _vp,
                                      ctypes.c_float, _vp, ctypes.c_int, _c_i64p, ctypes.c_float, _vp]),
    "dcpp_flux2_config_default": (None, [ctypes.POINTER(Flux2ConfigC)]),
    "dcpp_flux2_config_from_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(Flux2ConfigC)]),
    "dcpp_flux2_create": (ctypes.c_int, [_vp, ctypes.POINTER(Flux2ConfigC), ctypes.POINTER(_vp)]),
    "dcpp_flux2_destroy": (ctypes.c_int, [_vp]),
    "dcpp_flux2_set_param": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _c_i64p, _vp, ctypes.c_size_t]),
    "dcpp_flux2_missing": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, ctypes.c_size_t]),
    "dcpp_flux2_prepare": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]),
    "dcpp_flux2_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "dcpp_flux2_denoise_step": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp]),
    "dcpp_flux2_load_inputs": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "dcpp_flux2_prepare_ref": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int]),
    "dcpp_flux2_denoise_step_ref": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp]),
    "dcpp_flux2_load_inputs_ref": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "dcpp_flux2_set_timestep": (ctypes.c_int, [_vp, ctypes.c_float, ctypes.c_float]),
    "dcpp_flux2_run_resident": (ctypes.c_int, [_vp]),
    "dcpp_flux2_read_latents": (ctypes.c_int, [_vp, _vp]),
    "dcpp_flux2_launches_per_step": (ctypes.c_int, [_vp, _c_i64p]),
    "dcpp_flux2_set_profiling": (ctypes.c_int, [_vp, ctypes.c_int]),
    "dcpp_flux2_profile": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_double), _c_i64p]),
    "dcpp_flow_match_schedule": (ctypes.c_int, [ctypes.c_int, ctypes.c_float, _vp, _vp]),
    "dcpp_flow_match_config_default": (None, [ctypes.POINTER(FlowMatchConfigC)]),
    "dcpp_flow_match_schedule_ex": (ctypes.c_int, [ctypes.POINTER(FlowMatchConfigC), ctypes.c_int, ctypes.c_float,
                                                   _vp, _vp, _vp]),
    "dcpp_flux2_empirical_mu": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]),
    "dcpp_flux2_prepare_txt_ids": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _vp]),
    "dcpp_flux2_prepare_img_ids": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp]),
    "dcpp_flux2_prepare_ref_image_ids": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _vp, _vp]),
    "dcpp_tp_get_unique_id": (ctypes.c_int, [_vp]),
    "dcpp_tp_init": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    "dcpp_allreduce": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, ctypes.c_int]),
    "dcpp_flux2_set_tensor_parallel": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int]),
    "dcpp_flux2_set_tensor_split": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    "dcpp_flux2_shard": (ctypes.c_int, [_vp, _c_i64p, _c_i64p, _c_i64p, _c_i64p]),
    "dcpp_tp_plan_split": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int, _vp, _c_i64p]),
    "dcpp_flux2_create_host": (ctypes.c_int, [ctypes.POINTER(Flux2ConfigC), ctypes.POINTER(_vp)]),
    "dcpp_qwen3_config_default": (None, [ctypes.POINTER(Qwen3ConfigC)]),
    "dcpp_qwen3_config_from_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(Qwen3ConfigC)]),
    "dcpp_qwen3_create": (ctypes.c_int, [_vp, ctypes.POINTER(Qwen3ConfigC), ctypes.POINTER(_vp)]),
    "dcpp_qwen3_destroy": (ctypes.c_int, [_vp]),
    "dcpp_qwen3_set_param": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _c_i64p, _vp, ctypes.c_size_t]),
    "dcpp_qwen3_missing": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, ctypes.c_size_t]),
    "dcpp_qwen3_prepare": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                          ctypes.c_int]),
    "dcpp_qwen3_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "dcpp_qwen3_set_profiling": (ctypes.c_int, [_vp, ctypes.c_int]),
    "dcpp_qwen3_profile": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_double), _c_i64p]),
    "dcpp_qwen3_launches_per_step": (ctypes.c_int, [_vp, _c_i64p]),
    "dcpp_flux2_last_error": (ctypes.c_char_p, [_vp]),
    "dcpp_gguf_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.c_char_p, ctypes.c_size_t]),
    "dcpp_gguf_close": (None, [_vp]),
    "dcpp_gguf_info": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64), _c_i64p, _c_i64p]),
    "dcpp_gguf_tensor": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_int),
                                        ctypes.POINTER(ctypes.c_int), _c_i64p, ctypes.POINTER(ctypes.c_uint64),
                                        ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_vp)]),
    "dcpp_gguf_find_tensor": (ctypes.c_int64, [_vp, ctypes.c_char_p]),
    "dcpp_gguf_kv": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint64)]),
    "dcpp_gguf_get_int": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int64, _c_i64p]),
    "dcpp_gguf_get_float": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_double)]),
    "dcpp_gguf_get_string": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int64, ctypes.c_char_p, ctypes.c_size_t]),
    "dcpp_flux2_load_gguf": (ctypes.c_int, [_vp, _vp, _c_i64p, _c_i64p]),
    "dcpp_qwen3_load_gguf": (ctypes.c_int, [_vp, _vp, _c_i64p, _c_i64p]),
    "dcpp_flux2_from_pretrained": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "dcpp_vae_config_default": (None, [ctypes.POINTER(VAEConfigC)]),
    "dcpp_vae_config_from_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(VAEConfigC)]),
    "dcpp_vae_create": (ctypes.c_int, [_vp, ctypes.POINTER(VAEConfigC), ctypes.POINTER(_vp)]),
    "dcpp_vae_destroy": (ctypes.c_int, [_vp]),
    "dcpp_vae_set_param": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _c_i64p, _vp, ctypes.c_size_t]),
    "dcpp_vae_missing": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, ctypes.c_size_t]),
    "dcpp_vae_load_gguf": (ctypes.c_int, [_vp, _vp, _c_i64p, _c_i64p]),
    "dcpp_vae_from_pretrained": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "dcpp_vae_prepare": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]),
    "dcpp_vae_prepare_tiled": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int]),
    "dcpp_vae_decode": (ctypes.c_int, [_vp, _vp, _vp]),
    "dcpp_vae_set_profiling": (ctypes.c_int, [_vp, ctypes.c_int]),
    "dcpp_vae_profile": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double), _c_i64p]),
    "dcpp_vae_launches_per_step": (ctypes.c_int, [_vp, _c_i64p]),
    "dcpp_qwen3_from_pretrained": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "dcpp_flux2_read_param": (ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), _c_i64p, _c_i64p, _vp,
                                             ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load libdcpp_b200.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C diffusers-cpp_b200` "
                               "(or __graft_entry__.build()); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def exported_symbols() -> Iterable[str]:
    return _SIGNATURES.keys()


def _ptr(x) -> Optional[int]:
    """Address of a torch tensor / numpy array / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        assert x.is_contiguous(), "tensors passed to dcpp must be contiguous"
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        assert x.flags["C_CONTIGUOUS"]
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


class Context:
    """dcpp_ctx: one GPU, one stream."""

    def __init__(self, device: int = 0):
        h = _vp()
        st = lib().dcpp_init(device, ctypes.byref(h))
        if st != DCPP_OK:
            raise DcppError(st, f"dcpp_init({device}) failed")
        self.h = h
        self.device = device
        self._children = weakref.WeakSet()
        # With torch present the context runs on a torch stream, and every call
        # that touches device memory is ordered against torch's current stream
        # (_call): tensors torch has just produced (a .cuda() copy, a fill) are
        # complete before the library reads them, and torch work queued after
        # the call sees its results.
        self._stream = self._own_stream = None
        try:
            import torch
        except ImportError:
            torch = None
        if torch is not None and torch.cuda.is_available():
            self._own_stream = torch.cuda.Stream(device=device)
            self.check(lib().dcpp_set_stream(h, self._own_stream.cuda_stream), "set_stream")
            self._stream = self._own_stream

    def check(self, status: int, what: str = ""):
        if status != DCPP_OK:
            msg = lib().dcpp_last_error(self.h).decode()
            raise DcppError(status, f"{what}: {msg}" if what else msg)

    def close(self):
        if getattr(self, "h", None):
            for child in list(self._children):
                child.close()
            lib().dcpp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self):
        self.check(lib().dcpp_synchronize(self.h), "synchronize")

    def set_stream(self, stream_ptr: Optional[int]):
        """Run on an external cudaStream_t (None: back to the context's own)."""
        if stream_ptr:
            self.check(lib().dcpp_set_stream(self.h, stream_ptr), "set_stream")
            if self._own_stream is not None:
                import torch
                self._stream = torch.cuda.ExternalStream(stream_ptr, device=self.device)
        else:
            own = self._own_stream.cuda_stream if self._own_stream is not None else None
            self.check(lib().dcpp_set_stream(self.h, own), "set_stream")
            self._stream = self._own_stream

    def _call(self, fn, *args):
        """fn(*args) (a C entry point that reads or writes device memory),
        ordered with torch's current stream on both sides."""
        s = self._stream
        if s is None:
            return fn(*args)
        import torch
        cur = torch.cuda.current_stream(self.device)
        same = cur.cuda_stream == s.cuda_stream
        if not same:
            s.wait_stream(cur)
        st = fn(*args)
        if not same:
            cur.wait_stream(s)
        return st

    GEMM_AUTO, GEMM_SINGLE_SM, GEMM_PAIR = 0, 1, 2

    def set_gemm_kernel(self, kind: int):
        self.check(lib().dcpp_set_gemm_kernel(self.h, kind), "set_gemm_kernel")

    ATTN_AUTO, ATTN_ONE_TILE, ATTN_TWO_TILES = 0, 1, 2

    def set_attention_kernel(self, kind: int):
        self.check(lib().dcpp_set_attention_kernel(self.h, kind), "set_attention_kernel")

    def set_wait_timeout(self, seconds: float):
        """Limit of the cross-GPU barrier waits in plans prepared afterwards
        (0: the default 1 s)."""
        self.check(lib().dcpp_set_wait_timeout(self.h, float(seconds)), "set_wait_timeout")

    def tp_barrier_selftest(self, nranks: int, arrived_mask: int) -> int:
        """Run the barrier kernel as rank 0 of an emulated group on this GPU;
        returns the status (DCPP_ERR_TIMEOUT when a rank never arrives)."""
        return self._call(lib().dcpp_tp_barrier_selftest, self.h, nranks, arrived_mask)

    def inject_fault(self, name: Optional[str], nth: int = 1):
        lib().dcpp_inject_fault(self.h, name.encode() if name else None, nth)

    # op-level entry points (device pointers)
    def dequant(self, gtype: int, blocks, n: int, out):
        self.check(self._call(lib().dcpp_dequant, self.h, gtype, _ptr(blocks), n, _ptr(out)), "dequant")

    def dequant_bf16(self, gtype: int, blocks, n: int, out):
        self.check(self._call(lib().dcpp_dequant_bf16, self.h, gtype, _ptr(blocks), n, _ptr(out)), "dequant_bf16")

    def f32_to_bf16(self, x, n: int, out):
        self.check(self._call(lib().dcpp_f32_to_bf16, self.h, _ptr(x), n, _ptr(out)), "f32_to_bf16")

    def gemm(self, wtype: int, w, N: int, K: int, x_bf16, M: int, y):
        self.check(self._call(lib().dcpp_gemm, self.h, wtype, _ptr(w), N, K, _ptr(x_bf16), M, _ptr(y)), "gemm")

    def pack_weight(self, wtype: int, raw, N: int, K: int, out):
        self.check(self._call(lib().dcpp_pack_weight, self.h, wtype, _ptr(raw), N, K, _ptr(out)), "pack_weight")

    def gemm_packed(self, wtype: int, packed, N: int, K: int, x_bf16, M: int, y):
        self.check(self._call(lib().dcpp_gemm_packed, self.h, wtype, _ptr(packed), N, K, _ptr(x_bf16), M, _ptr(y)), "gemm_packed")

    def gemm_noalloc(self, wtype: int, w, N: int, K: int, x_bf16, M: int, y):
        """Like gemm(), but allocates no device memory: for callers whose
        device memory is owned by someone else or must not change mid-run
        (see dcpp_gemm_noalloc in include/dcpp.h for the limits)."""
        self.check(self._call(lib().dcpp_gemm_noalloc, self.h, wtype, _ptr(w), N, K, _ptr(x_bf16), M, _ptr(y)), "gemm_noalloc")

    def layernorm_mod(self, x, rows: int, D: int, shift, scale, eps: float, y):
        self.check(self._call(lib().dcpp_layernorm_mod, self.h, _ptr(x), rows, D, _ptr(shift), _ptr(scale), eps, _ptr(y)),
                   "layernorm_mod")

    def attention(self, qkv, B: int, S: int, H: int, norm_q, norm_k, eps: float, ids, axes_dims: Sequence[int],
                  theta: float, out):
        arr = (ctypes.c_int64 * len(axes_dims))(*axes_dims)
        self.check(self._call(lib().dcpp_attention, self.h, _ptr(qkv), B, S, H, 128, _ptr(norm_q), _ptr(norm_k), eps, _ptr(ids),
                                        len(axes_dims), arr, theta, _ptr(out)), "attention")

    # tensor parallelism
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
        st = lib().dcpp_tp_get_unique_id(buf)
        if st != DCPP_OK:
            raise DcppError(st, "dcpp_tp_get_unique_id")
        return buf.raw

    def tp_init(self, rank: int, nranks: int, uid: bytes):
        buf = ctypes.create_string_buffer(uid, NCCL_ID_BYTES)
        self.check(lib().dcpp_tp_init(self.h, rank, nranks, buf), "tp_init")

    def allreduce(self, buf, count: int, dtype: int = TYPE_F32):
        self.check(self._call(lib().dcpp_allreduce, self.h, _ptr(buf), count, dtype), "allreduce")


def packed_bytes(gtype: int, N: int, K: int) -> int:
    out = ctypes.c_size_t()
    st = lib().dcpp_packed_bytes(gtype, N, K, ctypes.byref(out))
    if st != DCPP_OK:
        raise DcppError(st, f"packed_bytes({gtype}, {N}, {K})")
    return out.value


def row_bytes(gtype: int, n: int) -> int:
    out = ctypes.c_size_t()
    st = lib().dcpp_row_bytes(gtype, n, ctypes.byref(out))
    if st != DCPP_OK:
        raise DcppError(st, f"row_bytes({gtype}, {n})")
    return out.value


def config_to_c(cfg) -> Flux2ConfigC:
    c = Flux2ConfigC()
    lib().dcpp_flux2_config_default(ctypes.byref(c))
    for k in ("patch_size", "in_channels", "num_layers", "num_single_layers", "attention_head_dim",
              "num_attention_heads", "joint_attention_dim", "timestep_guidance_channels", "rope_theta"):
        setattr(c, k, int(getattr(cfg, k)))
    c.out_channels = int(cfg.out_channels) if getattr(cfg, "out_channels", None) else -1
    c.mlp_ratio = float(cfg.mlp_ratio)
    c.eps = float(cfg.eps)
    c.guidance_embeds = 1 if cfg.guidance_embeds else 0
    c.n_axes = len(cfg.axes_dims_rope)
    for i, d in enumerate(cfg.axes_dims_rope):
        c.axes_dims_rope[i] = int(d)
    return c


class Flux2Model:
    """dcpp_flux2: Flux2Transformer2DModel on one GPU (or one TP rank).

    ``ctx=None`` makes a host-only model (dcpp_flux2_create_host): parameters
    are assembled and sharded exactly as on a device, but stay on the host
    (``read_param``) and the model cannot execute."""

    def __init__(self, ctx: Optional[Context], cfg, tp_rank: int = 0, tp_size: int = 1, tp_split=None):
        self.ctx = ctx
        self.cfg = cfg
        c = config_to_c(cfg)
        h = _vp()
        if ctx is None:
            st = lib().dcpp_flux2_create_host(ctypes.byref(c), ctypes.byref(h))
            if st != DCPP_OK:
                raise DcppError(st, "flux2_create_host")
        else:
            ctx.check(lib().dcpp_flux2_create(ctx.h, ctypes.byref(c), ctypes.byref(h)), "flux2_create")
            ctx._children.add(self)
        self.h = h
        if tp_split is not None:
            arr = (ctypes.c_float * tp_size)(*[float(f) for f in tp_split])
            self._check(lib().dcpp_flux2_set_tensor_split(h, tp_rank, tp_size, arr), "set_tensor_split")
        elif tp_size > 1:
            self._check(lib().dcpp_flux2_set_tensor_parallel(h, tp_rank, tp_size), "set_tensor_parallel")

    @classmethod
    def from_pretrained(cls, ctx: Context, path):
        """config.json + the GGUF file of a transformer folder
        (Flux2KleinPipeline::from_pretrained's "<model>/transformer")."""
        self = cls.__new__(cls)
        self.ctx = ctx
        c = Flux2ConfigC()
        ctx.check(lib().dcpp_flux2_config_from_file(os.path.join(os.fspath(path), "config.json").encode(),
                                                    ctypes.byref(c)), "config_from_file")
        self.cfg = c
        h = _vp()
        ctx.check(lib().dcpp_flux2_from_pretrained(ctx.h, os.fspath(path).encode(), ctypes.byref(h)), "from_pretrained")
        ctx._children.add(self)
        self.h = h
        return self

    def _check(self, status: int, what: str = ""):
        if status != DCPP_OK:
            msg = lib().dcpp_flux2_last_error(self.h).decode()
            raise DcppError(status, f"{what}: {msg}" if what else msg)

    def _run(self, fn, *args):
        # host-only models have no context (their compute calls fail in the library)
        return self.ctx._call(fn, *args) if self.ctx is not None else fn(*args)

    def shard(self):
        """(first head, heads, first MLP feature, MLP features) of this rank."""
        v = [ctypes.c_int64() for _ in range(4)]
        self._check(lib().dcpp_flux2_shard(self.h, *[ctypes.byref(x) for x in v]), "shard")
        return tuple(x.value for x in v)

    def read_param(self, name: str):
        """(ggml type, (rows, cols), uint8 array) of an assembled parameter."""
        t, r, c, n = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_size_t()
        self._check(lib().dcpp_flux2_read_param(self.h, name.encode(), ctypes.byref(t), ctypes.byref(r),
                                                ctypes.byref(c), None, 0, ctypes.byref(n)), f"read_param({name})")
        buf = np.empty(n.value, dtype=np.uint8)
        self._check(lib().dcpp_flux2_read_param(self.h, name.encode(), None, None, None, buf.ctypes.data, buf.nbytes,
                                                ctypes.byref(n)), f"read_param({name})")
        return t.value, (r.value, c.value), buf

    def close(self):
        if getattr(self, "h", None):
            lib().dcpp_flux2_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_param(self, name: str, gtype: int, shape: Sequence[int], data):
        """`data`: bytes-like / numpy uint8 array / CPU torch uint8 tensor holding raw GGUF bytes."""
        if hasattr(data, "numpy"):
            data = data.contiguous().cpu().numpy()
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8))
        shp = (ctypes.c_int64 * len(shape))(*shape)
        self._check(lib().dcpp_flux2_set_param(self.h, name.encode(), gtype, len(shape), shp, arr.ctypes.data,
                                                  arr.nbytes), f"set_param({name})")

    def load_params(self, params):
        for name, (gtype, shape, data) in params.items():
            self.set_param(name, gtype, shape, data)

    def load_gguf(self, source):
        """Bind every tensor of a GGUF checkpoint (a GGUFFile, a .gguf path or a
        folder holding one); returns (tensors bound, tensors the model did not
        know).  Raises if a parameter is not in the file."""
        f = source if isinstance(source, GGUFFile) else GGUFFile(source)
        nb, nu = ctypes.c_int64(), ctypes.c_int64()
        self._check(lib().dcpp_flux2_load_gguf(self.h, f.h, ctypes.byref(nb), ctypes.byref(nu)), "load_gguf")
        return nb.value, nu.value

    def missing(self):
        n = ctypes.c_int()
        buf = ctypes.create_string_buffer(512)
        self._check(lib().dcpp_flux2_missing(self.h, ctypes.byref(n), buf, 512), "missing")
        return n.value, buf.value.decode()

    def prepare(self, batch: int, n_img: int, n_txt: int, use_graph: bool = True, n_ref: int = 0):
        """Plan batch x (n_img + n_ref + n_txt) tokens; n_ref reference-image
        tokens follow the latent tokens (dcpp_flux2_prepare_ref)."""
        if n_ref:
            self._check(lib().dcpp_flux2_prepare_ref(self.h, batch, n_img, n_ref, n_txt, 1 if use_graph else 0),
                        "prepare_ref")
        else:
            self._check(lib().dcpp_flux2_prepare(self.h, batch, n_img, n_txt, 1 if use_graph else 0), "prepare")

    def forward(self, hidden, encoder, timestep, img_ids, txt_ids, out, guidance=None):
        self._check(self._run(lib().dcpp_flux2_forward, self.h, _ptr(hidden), _ptr(encoder), _ptr(timestep), _ptr(img_ids),
                                                _ptr(txt_ids), _ptr(guidance), _ptr(out)), "forward")

    def denoise_step(self, latents, encoder, timestep, dt: float, img_ids, txt_ids, latents_out,
                     image_latents=None, image_latent_ids=None):
        """Flux2KleinPipeline::denoise for one step; with image_latents (and
        their ids) the reference tokens join the image stream and only the
        latent tokens are integrated (dcpp_flux2_denoise_step_ref)."""
        if image_latents is not None or image_latent_ids is not None:
            self._check(self._run(lib().dcpp_flux2_denoise_step_ref, self.h, _ptr(latents), _ptr(image_latents),
                                  _ptr(image_latent_ids), _ptr(encoder), _ptr(timestep), float(dt), _ptr(img_ids),
                                  _ptr(txt_ids), _ptr(latents_out)), "denoise_step_ref")
            return
        self._check(self._run(lib().dcpp_flux2_denoise_step, self.h, _ptr(latents), _ptr(encoder), _ptr(timestep), float(dt),
                                                     _ptr(img_ids), _ptr(txt_ids), _ptr(latents_out)), "denoise_step")

    def load_inputs(self, latents, encoder, img_ids, txt_ids, image_latents=None, image_latent_ids=None):
        if image_latents is not None or image_latent_ids is not None:
            self._check(self._run(lib().dcpp_flux2_load_inputs_ref, self.h, _ptr(latents), _ptr(image_latents),
                                  _ptr(image_latent_ids), _ptr(encoder), _ptr(img_ids), _ptr(txt_ids)),
                        "load_inputs_ref")
            return
        self._check(self._run(lib().dcpp_flux2_load_inputs, self.h, _ptr(latents), _ptr(encoder), _ptr(img_ids),
                                                    _ptr(txt_ids)), "load_inputs")

    def set_timestep(self, timestep: float, dt: float):
        self._check(lib().dcpp_flux2_set_timestep(self.h, float(timestep), float(dt)), "set_timestep")

    def run_resident(self):
        self._check(self._run(lib().dcpp_flux2_run_resident, self.h), "run_resident")

    def read_latents(self, out):
        self._check(self._run(lib().dcpp_flux2_read_latents, self.h, _ptr(out)), "read_latents")

    PROFILE_KINDS = {"gemm": 0, "attention": 1, "norm": 2, "gemv": 3, "dequant": 4, "other": 5, "allreduce": 6}

    def set_profiling(self, on: bool):
        self._check(lib().dcpp_flux2_set_profiling(self.h, 1 if on else 0), "set_profiling")

    def profile(self, kind: str):
        ms, fl, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
        self._check(lib().dcpp_flux2_profile(self.h, self.PROFILE_KINDS[kind], ctypes.byref(ms), ctypes.byref(fl),
                                                ctypes.byref(n)), "profile")
        return ms.value, fl.value, n.value

    def launches_per_step(self) -> int:
        v = ctypes.c_int64()
        self._check(lib().dcpp_flux2_launches_per_step(self.h, ctypes.byref(v)), "launches_per_step")
        return v.value


GGUF_VALUE_TYPES = {0: "u8", 1: "i8", 2: "u16", 3: "i16", 4: "u32", 5: "i32", 6: "f32", 7: "bool", 8: "string",
                    9: "array", 10: "u64", 11: "i64", 12: "f64"}


class GGUFFile:
    """dcpp_gguf: a memory-mapped GGUF checkpoint (a .gguf file, or a component
    folder holding one), as GGUFLoaderVisitor opens it."""

    def __init__(self, path):
        h = _vp()
        err = ctypes.create_string_buffer(2048)
        st = lib().dcpp_gguf_open(os.fspath(path).encode(), ctypes.byref(h), err, len(err))
        if st != DCPP_OK:
            raise DcppError(st, err.value.decode())
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().dcpp_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def info(self):
        v, a, d = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint64()
        nt, nk = ctypes.c_int64(), ctypes.c_int64()
        st = lib().dcpp_gguf_info(self.h, ctypes.byref(v), ctypes.byref(a), ctypes.byref(d), ctypes.byref(nt),
                                  ctypes.byref(nk))
        if st != DCPP_OK:
            raise DcppError(st, "gguf_info")
        return {"version": v.value, "alignment": a.value, "data_offset": d.value, "n_tensors": nt.value,
                "n_kv": nk.value}

    def tensor(self, i: int):
        """dict(name, type, ne (ggml order, n_dims entries), offset, nbytes, data address)."""
        name, t, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        ne = (ctypes.c_int64 * 4)()
        off, nb, data = ctypes.c_uint64(), ctypes.c_uint64(), _vp()
        st = lib().dcpp_gguf_tensor(self.h, i, ctypes.byref(name), ctypes.byref(t), ctypes.byref(nd), ne,
                                    ctypes.byref(off), ctypes.byref(nb), ctypes.byref(data))
        if st != DCPP_OK:
            raise DcppError(st, f"gguf_tensor({i})")
        return {"name": name.value.decode(), "type": t.value, "ne": tuple(ne[:nd.value]), "offset": off.value,
                "nbytes": nb.value, "data": data.value}

    def tensors(self):
        return [self.tensor(i) for i in range(self.info()["n_tensors"])]

    def find(self, name: str) -> int:
        return int(lib().dcpp_gguf_find_tensor(self.h, name.encode()))

    def tensor_bytes(self, name: str) -> np.ndarray:
        i = self.find(name)
        if i < 0:
            raise KeyError(name)
        t = self.tensor(i)
        return np.ctypeslib.as_array((ctypes.c_uint8 * t["nbytes"]).from_address(t["data"])).copy()

    def _get(self, key: str, vtype: int, index: int):
        k = key.encode()
        if vtype == 8:
            cap = 256
            while True:
                buf = ctypes.create_string_buffer(cap)
                st = lib().dcpp_gguf_get_string(self.h, k, index, buf, cap)
                if st == DCPP_OK:
                    return buf.value.decode("utf-8", errors="surrogateescape")
                if cap > (1 << 26):
                    raise DcppError(st, f"gguf_get_string({key})")
                cap *= 4
        if vtype in (6, 12):
            out = ctypes.c_double()
            st = lib().dcpp_gguf_get_float(self.h, k, index, ctypes.byref(out))
        else:
            out = ctypes.c_int64()
            st = lib().dcpp_gguf_get_int(self.h, k, index, ctypes.byref(out))
        if st != DCPP_OK:
            raise DcppError(st, f"gguf_get({key})")
        return bool(out.value) if vtype == 7 else out.value

    def metadata(self):
        """{key: (type name, value)}; arrays as ("array[<elem type>]", list)."""
        out = {}
        for i in range(self.info()["n_kv"]):
            key, t, et, n = ctypes.c_char_p(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint64()
            st = lib().dcpp_gguf_kv(self.h, i, ctypes.byref(key), ctypes.byref(t), ctypes.byref(et), ctypes.byref(n))
            if st != DCPP_OK:
                raise DcppError(st, f"gguf_kv({i})")
            k = key.value.decode()
            if t.value == 9:
                out[k] = (f"array[{GGUF_VALUE_TYPES.get(et.value, et.value)}]",
                          [self._get(k, et.value, j) for j in range(n.value)])
            else:
                out[k] = (GGUF_VALUE_TYPES.get(t.value, t.value), self._get(k, t.value, -1))
        return out


def tp_plan_split(units: int, nranks: int, ratios=None):
    """The sharding planner's split of `units` over nranks (dcpp_tp_plan_split)."""
    out = (ctypes.c_int64 * nranks)()
    arr = (ctypes.c_float * nranks)(*[float(f) for f in ratios]) if ratios is not None else None
    st = lib().dcpp_tp_plan_split(units, nranks, arr, out)
    if st != DCPP_OK:
        raise DcppError(st, "tp_plan_split")
    return list(out)


def flow_match_schedule(n: int, shift: float = 1.0):
    ts = np.zeros(n, dtype=np.float32)
    sg = np.zeros(n + 1, dtype=np.float32)
    st = lib().dcpp_flow_match_schedule(n, shift, ts.ctypes.data, sg.ctypes.data)
    if st != DCPP_OK:
        raise DcppError(st, "flow_match_schedule")
    return ts, sg


class FlowMatchEulerDiscreteScheduler:
    """The reference scheduler's constructor options and schedule(n, mu,
    sigmas) (FlowMatchEulerDiscreteScheduler.hpp:11-23), through
    dcpp_flow_match_schedule_ex.  schedule returns (timesteps[n],
    sigmas[n + 1]) as float32 arrays."""

    def __init__(self, num_train_timesteps=1000, shift=1.0, use_dynamic_shifting=False, shift_terminal=None,
                 invert_sigmas=False, time_shift_type="exponential"):
        if time_shift_type not in ("exponential", "linear"):
            raise DcppError(DCPP_ERR_INVALID_ARG, f"unsupported time_shift_type: {time_shift_type}")
        self.config = FlowMatchConfigC()
        lib().dcpp_flow_match_config_default(ctypes.byref(self.config))
        self.config.num_train_timesteps = int(num_train_timesteps)
        self.config.shift = float(shift)
        self.config.use_dynamic_shifting = int(bool(use_dynamic_shifting))
        self.config.has_shift_terminal = int(shift_terminal is not None)
        self.config.shift_terminal = float(shift_terminal) if shift_terminal is not None else 0.0
        self.config.invert_sigmas = int(bool(invert_sigmas))
        self.config.time_shift_type = 1 if time_shift_type == "linear" else 0

    def schedule(self, n: int, mu: float = 0.0, sigmas=None):
        ts = np.zeros(max(n, 0), dtype=np.float32)
        sg = np.zeros(max(n, 0) + 1, dtype=np.float32)
        base = None
        if sigmas is not None:
            base = np.ascontiguousarray(np.asarray(sigmas, dtype=np.float32))
            if base.size != n:
                raise DcppError(DCPP_ERR_INVALID_ARG, "sigmas must have n entries")
        st = lib().dcpp_flow_match_schedule_ex(ctypes.byref(self.config), n, float(mu),
                                               base.ctypes.data if base is not None else None, ts.ctypes.data,
                                               sg.ctypes.data)
        if st != DCPP_OK:
            raise DcppError(st, "FlowMatchEulerDiscreteScheduler.schedule")
        return ts, sg


def prepare_txt_ids(batch: int, seq_len: int):
    """The pipeline's txt_ids [batch, seq_len, 4] int32 (dcpp_flux2_prepare_txt_ids)."""
    out = np.zeros((batch, seq_len, 4), dtype=np.int32)
    st = lib().dcpp_flux2_prepare_txt_ids(batch, seq_len, out.ctypes.data)
    if st != DCPP_OK:
        raise DcppError(st, "prepare_txt_ids")
    return out


def prepare_img_ids(batch: int, packed_h: int, packed_w: int):
    """The pipeline's img_ids [batch, packed_h * packed_w, 4] int32."""
    out = np.zeros((batch, packed_h * packed_w, 4), dtype=np.int32)
    st = lib().dcpp_flux2_prepare_img_ids(batch, packed_h, packed_w, out.ctypes.data)
    if st != DCPP_OK:
        raise DcppError(st, "prepare_img_ids")
    return out


def prepare_ref_image_ids(batch: int, packed_sizes):
    """The pipeline's image_latent_ids [batch, sum h*w, 4] int32 for reference
    images of packed sizes [(h, w), ...] (image size / (VAE scale factor * 2))."""
    hw = np.ascontiguousarray(np.asarray(packed_sizes, dtype=np.int64).reshape(-1, 2))
    tokens = int((hw[:, 0] * hw[:, 1]).sum()) if hw.size else 0
    out = np.zeros((batch, tokens, 4), dtype=np.int32)
    st = lib().dcpp_flux2_prepare_ref_image_ids(batch, hw.shape[0], hw.ctypes.data if hw.size else None,
                                                out.ctypes.data)
    if st != DCPP_OK:
        raise DcppError(st, "prepare_ref_image_ids")
    return out


def flux2_empirical_mu(image_seq_len: int, num_steps: int) -> float:
    """The Flux2 Klein pipeline's compute_empirical_mu (dynamic-shift mu)."""
    mu = ctypes.c_float()
    st = lib().dcpp_flux2_empirical_mu(int(image_seq_len), int(num_steps), ctypes.byref(mu))
    if st != DCPP_OK:
        raise DcppError(st, "flux2_empirical_mu")
    return mu.value


def qwen3_config_to_c(cfg) -> Qwen3ConfigC:
    c = Qwen3ConfigC()
    lib().dcpp_qwen3_config_default(ctypes.byref(c))
    for k in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
              "num_key_value_heads", "head_dim"):
        setattr(c, k, int(getattr(cfg, k)))
    c.rms_norm_eps = float(cfg.rms_norm_eps)
    c.rope_theta = float(cfg.rope_theta)
    return c


class Qwen3Model:
    """dcpp_qwen3: the Qwen3 text-encoder prefill (Qwen3Model::forward) on one GPU."""

    def __init__(self, ctx: Context, cfg):
        self.ctx = ctx
        self.cfg = cfg
        c = qwen3_config_to_c(cfg)
        h = _vp()
        ctx.check(lib().dcpp_qwen3_create(ctx.h, ctypes.byref(c), ctypes.byref(h)), "qwen3_create")
        ctx._children.add(self)
        self.h = h
        self.n_taps = 0

    @classmethod
    def from_pretrained(cls, ctx: Context, path):
        """config.json + the GGUF file of a text-encoder folder
        (Flux2KleinPipeline::from_pretrained's "<model>/text_encoder")."""
        self = cls.__new__(cls)
        self.ctx = ctx
        c = Qwen3ConfigC()
        ctx.check(lib().dcpp_qwen3_config_from_file(os.path.join(os.fspath(path), "config.json").encode(),
                                                    ctypes.byref(c)), "config_from_file")
        self.cfg = c
        h = _vp()
        ctx.check(lib().dcpp_qwen3_from_pretrained(ctx.h, os.fspath(path).encode(), ctypes.byref(h)), "from_pretrained")
        ctx._children.add(self)
        self.h = h
        self.n_taps = 0
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().dcpp_qwen3_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_param(self, name: str, gtype: int, shape: Sequence[int], data):
        if hasattr(data, "numpy"):
            data = data.contiguous().cpu().numpy()
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8))
        shp = (ctypes.c_int64 * len(shape))(*shape)
        self.ctx.check(lib().dcpp_qwen3_set_param(self.h, name.encode(), gtype, len(shape), shp, arr.ctypes.data,
                                                  arr.nbytes), f"set_param({name})")

    def load_params(self, params):
        for name, (gtype, shape, data) in params.items():
            self.set_param(name, gtype, shape, data)

    def load_gguf(self, source):
        """As Flux2Model.load_gguf, for the text encoder's checkpoint."""
        f = source if isinstance(source, GGUFFile) else GGUFFile(source)
        nb, nu = ctypes.c_int64(), ctypes.c_int64()
        self.ctx.check(lib().dcpp_qwen3_load_gguf(self.h, f.h, ctypes.byref(nb), ctypes.byref(nu)), "load_gguf")
        return nb.value, nu.value

    def missing(self):
        n = ctypes.c_int()
        buf = ctypes.create_string_buffer(512)
        self.ctx.check(lib().dcpp_qwen3_missing(self.h, ctypes.byref(n), buf, 512), "missing")
        return n.value, buf.value.decode()

    def prepare(self, batch: int, seq: int, taps: Sequence[int] = (), use_graph: bool = True):
        arr = (ctypes.c_int * max(len(taps), 1))(*taps)
        self.ctx.check(lib().dcpp_qwen3_prepare(self.h, batch, seq, len(taps), arr, 1 if use_graph else 0), "prepare")
        self.n_taps = len(taps)

    def forward(self, input_ids, last_hidden=None, taps=None, attention_mask=None):
        """input_ids [B, S] int32; attention_mask [B, S] f32 (1 attend, 0 padding)
        or None; last_hidden [B, S, D] f32; taps [B, S, n_taps * D] f32."""
        self.ctx.check(self.ctx._call(lib().dcpp_qwen3_forward, self.h, _ptr(input_ids), _ptr(attention_mask), _ptr(last_hidden),
                                                _ptr(taps)), "forward")

    def set_profiling(self, on: bool):
        self.ctx.check(lib().dcpp_qwen3_set_profiling(self.h, 1 if on else 0), "set_profiling")

    def profile(self, kind: str):
        ms, fl, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
        self.ctx.check(lib().dcpp_qwen3_profile(self.h, Flux2Model.PROFILE_KINDS[kind], ctypes.byref(ms),
                                                ctypes.byref(fl), ctypes.byref(n)), "profile")
        return ms.value, fl.value, n.value

    def launches_per_step(self) -> int:
        v = ctypes.c_int64()
        self.ctx.check(lib().dcpp_qwen3_launches_per_step(self.h, ctypes.byref(v)), "launches_per_step")
        return v.value


def vae_config_to_c(cfg) -> VAEConfigC:
    """VAEConfigC from an object with AutoencoderKLFlux2::Config's field names."""
    c = VAEConfigC()
    lib().dcpp_vae_config_default(ctypes.byref(c))
    for k in ("in_channels", "out_channels", "layers_per_block", "latent_channels", "norm_num_groups"):
        if hasattr(cfg, k):
            setattr(c, k, int(getattr(cfg, k)))
    ch = list(cfg.block_out_channels)
    c.n_blocks = len(ch)
    for i, v in enumerate(ch):
        c.block_out_channels[i] = int(v)
    for k in ("use_post_quant_conv", "mid_block_add_attention"):
        if hasattr(cfg, k):
            setattr(c, k, 1 if getattr(cfg, k) else 0)
    if hasattr(cfg, "batch_norm_eps"):
        c.batch_norm_eps = float(cfg.batch_norm_eps)
    return c


class VAEModel:
    """dcpp_vae: the Flux2 VAE decode (Flux2KleinPipeline::decode) on one GPU."""

    PROFILE_KINDS = Flux2Model.PROFILE_KINDS

    def __init__(self, ctx: Context, cfg):
        self.ctx = ctx
        self.cfg = cfg
        c = vae_config_to_c(cfg)
        h = _vp()
        ctx.check(lib().dcpp_vae_create(ctx.h, ctypes.byref(c), ctypes.byref(h)), "vae_create")
        ctx._children.add(self)
        self.h = h

    @classmethod
    def from_pretrained(cls, ctx: Context, path):
        """config.json + the GGUF file of the pipeline's vae folder."""
        self = cls.__new__(cls)
        self.ctx = ctx
        c = VAEConfigC()
        ctx.check(lib().dcpp_vae_config_from_file(os.path.join(os.fspath(path), "config.json").encode(),
                                                  ctypes.byref(c)), "config_from_file")
        self.cfg = c
        h = _vp()
        ctx.check(lib().dcpp_vae_from_pretrained(ctx.h, os.fspath(path).encode(), ctypes.byref(h)), "from_pretrained")
        ctx._children.add(self)
        self.h = h
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().dcpp_vae_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_param(self, name: str, gtype: int, shape: Sequence[int], data):
        if hasattr(data, "numpy"):
            data = data.contiguous().cpu().numpy()
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8))
        shp = (ctypes.c_int64 * len(shape))(*shape)
        self.ctx.check(lib().dcpp_vae_set_param(self.h, name.encode(), gtype, len(shape), shp, arr.ctypes.data,
                                                arr.nbytes), f"set_param({name})")

    def load_params(self, params):
        for name, (gtype, shape, data) in params.items():
            self.set_param(name, gtype, shape, data)

    def load_gguf(self, source):
        f = source if isinstance(source, GGUFFile) else GGUFFile(source)
        nb, nu = ctypes.c_int64(), ctypes.c_int64()
        self.ctx.check(lib().dcpp_vae_load_gguf(self.h, f.h, ctypes.byref(nb), ctypes.byref(nu)), "load_gguf")
        return nb.value, nu.value

    def missing(self):
        n = ctypes.c_int()
        buf = ctypes.create_string_buffer(512)
        self.ctx.check(lib().dcpp_vae_missing(self.h, ctypes.byref(n), buf, 512), "missing")
        return n.value, buf.value.decode()

    def prepare(self, batch: int, packed_h: int, packed_w: int, use_graph: bool = True, tile_size: int = 0):
        """tile_size > 0: the tiled decode (decode_tiled) with tiles of that many pixels."""
        if tile_size:
            self.ctx.check(lib().dcpp_vae_prepare_tiled(self.h, batch, packed_h, packed_w, tile_size,
                                                        1 if use_graph else 0), "prepare_tiled")
        else:
            self.ctx.check(lib().dcpp_vae_prepare(self.h, batch, packed_h, packed_w, 1 if use_graph else 0), "prepare")

    def decode(self, latents, image):
        """latents [B, ph*pw, 4*latent_channels] f32 -> image [B, out_channels, H, W] f32."""
        self.ctx.check(self.ctx._call(lib().dcpp_vae_decode, self.h, _ptr(latents), _ptr(image)), "decode")

    def set_profiling(self, on: bool):
        self.ctx.check(lib().dcpp_vae_set_profiling(self.h, 1 if on else 0), "set_profiling")

    def profile(self, kind: str):
        ms, fl, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
        self.ctx.check(lib().dcpp_vae_profile(self.h, self.PROFILE_KINDS[kind], ctypes.byref(ms), ctypes.byref(fl),
                                              ctypes.byref(n)), "profile")
        return ms.value, fl.value, n.value

    def launches_per_step(self) -> int:
        v = ctypes.c_int64()
        self.ctx.check(lib().dcpp_vae_launches_per_step(self.h, ctypes.byref(v)), "launches_per_step")
        return v.value
