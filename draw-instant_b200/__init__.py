"""draw-instant B200: host-side binding of libdi.so (the sm_100a kernels of the SD-Turbo denoising hot path).

The reference's host is JavaScript calling WebGPU; this package is the Python mirror of that host
interface over libdi's C ABI (ctypes, plain device pointers).  Device memory and streams come from
PyTorch tensors (plumbing only): every op takes CUDA tensors and passes their data pointers.

Modules:
  ops       the wgsl-ops.js closures (op(ctx, ...) -> dispatch(...)), fp32, reference layouts
  blocks    the fused blocks (resnet, conv, groupnorm, attn, cross-attn, block-full, tembed) and
            their runXBench drivers with the reference's result schema
  unet      the SD-Turbo U-Net plan (CUDA-graph replay of the whole forward)

There is no CPU fallback: importing this package on a machine without a CUDA device works (so the
library can be inspected), but every compute call raises when libdi.so or the GPU is missing.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ["DI_LIB"]) if os.environ.get("DI_LIB") else PKG_DIR / "libdi.so"  # DI_LIB: diagnostics

DI_OK, DI_EINVAL, DI_ECUDA, DI_ENOMEM, DI_EUNSUPPORTED, DI_EFAULT = 0, -1, -2, -3, -4, -5
DI_F32, DI_F16, DI_BF16 = 0, 1, 2

UNARY = {"Sigmoid": 0, "Sqrt": 1, "Neg": 2, "Abs": 3, "Sin": 4, "Cos": 5, "Exp": 6, "Log": 7, "SiLU": 8,
         "GELU": 9, "Erf": 10}
BINARY = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3, "Pow": 4, "Max": 5, "Min": 6}

_P = ctypes.c_void_p
_I = ctypes.c_int
_U = ctypes.c_uint32
_F = ctypes.c_float
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/di.h
SIGNATURES = {
    "di_init": (_I, [_I, ctypes.POINTER(_P)]),
    "di_destroy": (None, [_P]),
    "di_set_stream": (_I, [_P, _P]),
    "di_get_stream": (_P, [_P]),
    "di_buf_alloc": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "di_buf_free": (_I, [_P]),
    "di_buf_ptr": (_P, [_P]),
    "di_buf_size": (_SZ, [_P]),
    "di_buf_upload": (_I, [_P, _P, _SZ, _SZ]),
    "di_buf_download": (_I, [_P, _P, _SZ, _SZ]),
    "di_wait": (_I, [_P]),
    "di_last_error": (ctypes.c_char_p, [_P]),
    "di_device_fault": (_I, [_P]),
    "di_clear_fault": (_I, [_P]),
    "di_debug_gemm_trace": (_I, [_P, _I]),
    "di_debug_wait_timeout": (_I, [_P, _I]),
    "di_f16_bytes_to_f32": (_I, [_P, _P, _P, _SZ]),
    "di_unary": (_I, [_P, _I, _P, _P, _U]),
    "di_binary": (_I, [_P, _I, _P, _U, _P, _U, _P, _U]),
    "di_binary_bcast": (_I, [_P, _I, _P, _P, _P, _P]),
    "di_affine_bcast": (_I, [_P, _P, _P, _P, _P, _P]),
    "di_softmax": (_I, [_P, _P, _P, _P]),
    "di_instance_norm": (_I, [_P, _P, _P, _P, _P, _P]),
    "di_group_norm": (_I, [_P, _P, _P, _P, _P, _P, _I]),
    "di_layer_norm": (_I, [_P, _P, _P, _P, _P, _P]),
    "di_matmul": (_I, [_P, _P, _P, _P, _P, _U]),
    "di_gemm": (_I, [_P, _P, _P, _P, _P, _P]),
    "di_conv": (_I, [_P, _P, _P, _P, _P, _P, _U]),
    "di_resize_nearest": (_I, [_P, _P, _P, _P]),
    "di_reduce_mean": (_I, [_P, _P, _P, _P]),
    "di_transpose": (_I, [_P, _P, _P, _P]),
    "di_pow_scalar": (_I, [_P, _P, _P, _F, _U]),
    "di_slice": (_I, [_P, _P, _P, _P]),
    "di_concat_copy": (_I, [_P, _P, _P, _P]),
    "di_group_norm_nhwc": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _F, _P, _P, _I, _P]),
    "di_group_norm_nhwc_noalloc": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _F, _P, _P, _I, _P]),
    "di_linear": (_I, [_P, _I, _P, _I, _P, _I, _I, _P, _I, _P, _P, _P]),
    "di_linear_geglu": (_I, [_P, _I, _P, _I, _I, _P, _I, _P, _P]),
    "di_conv3x3_nhwc": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P]),
    "di_pack_conv3x3": (_I, [_P, _I, _P, _I, _I, _P]),
    "di_conv3x3_nhwc_act": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _I, _P]),
    "di_gn_table_nhwc": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _F, _P, _P, _P]),
    "di_conv3x3_nhwc_gn": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _I, _P]),
    "di_attention": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I]),
    "di_tembed": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _I, _P]),
    "di_synth_uniform": (None, [ctypes.c_uint64, ctypes.c_char_p, _SZ, _F, _P]),
    "di_synth_normal": (None, [ctypes.c_uint64, ctypes.c_char_p, _SZ, _F, _F, _P]),
    "di_euler_sigmas": (_I, [_I, _P, _P]),
    "di_unet_create": (_I, [_P, _I, _I, _I, _I, ctypes.c_uint64, _P, _P, ctypes.POINTER(_P)]),
    "di_unet_io": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "di_unet_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "di_unet_ops": (_I, [_P, ctypes.POINTER(_I), _P, _P, _P, _P]),
    "di_unet_profile": (_I, [_P, _I, _P]),
    "di_unet_profile_kind": (_I, [_P, _I, _I, ctypes.POINTER(_F)]),
    "di_unet_forward": (_I, [_P]),
    "di_unet_forward_host": (_I, [_P, _P, _P, _P, _P]),
    "di_unet_destroy": (None, [_P]),
    "di_vae_create": (_I, [_P, _I, _I, _I, ctypes.c_uint64, _P, _P, ctypes.POINTER(_P)]),
    "di_vae_io": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "di_vae_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "di_vae_ops": (_I, [_P, ctypes.POINTER(_I), _P, _P, _P, _P]),
    "di_vae_profile_kind": (_I, [_P, _I, _I, ctypes.POINTER(_F)]),
    "di_vae_forward": (_I, [_P]),
    "di_vae_forward_host": (_I, [_P, _P, _P]),
    "di_vae_destroy": (None, [_P]),
    "di_vae_debug_copy": (_I, [_P, _I, _SZ, _P, _SZ]),
    "di_linear_act": (_I, [_P, _I, _P, _I, _I, _P, _I, _P, _P, _I, _P]),
    "di_attention_causal": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I]),
    "di_unet_sched": (_I, [_P, ctypes.c_double, ctypes.c_double, ctypes.POINTER(_P)]),
    "di_text_create": (_I, [_P, _I, _I, _I, ctypes.c_uint64, _P, _P, ctypes.POINTER(_P)]),
    "di_text_io": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "di_text_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "di_text_ops": (_I, [_P, ctypes.POINTER(_I), _P, _P, _P, _P]),
    "di_text_forward": (_I, [_P]),
    "di_text_forward_host": (_I, [_P, _P, _P]),
    "di_text_destroy": (None, [_P]),
    "di_t2i_create": (_I, [_P, _I, _I, _I, _I, ctypes.c_uint64, _P, _P, ctypes.POINTER(_P)]),
    "di_t2i_io": (_I, [_P] + [ctypes.POINTER(_P)] * 5),
    "di_t2i_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ), ctypes.POINTER(_F)]),
    "di_t2i_forward": (_I, [_P, _I]),
    "di_t2i_forward_host": (_I, [_P, _P, _P, _P]),
    "di_t2i_destroy": (None, [_P]),
    "di_resnet_block_create": (_I, [_P, _I, _I, _I, _I, _I, ctypes.c_uint64, _F, _I, _P, _P, ctypes.POINTER(_P)]),
    "di_resnet_block_io": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "di_resnet_block_run": (_I, [_P]),
    "di_resnet_block_destroy": (None, [_P]),
    "di_transformer_block_create": (_I, [_P, _I, _I, _I, _I, _I, ctypes.c_uint64, _P, _P, ctypes.POINTER(_P)]),
    "di_transformer_block_io": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "di_transformer_block_run": (_I, [_P]),
    "di_transformer_block_destroy": (None, [_P]),
}

WEIGHT_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_float),
                             ctypes.c_void_p)

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libdi.so from the package directory (built by build.py); raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python draw-instant_b200/build.py` (no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class DIError(RuntimeError):
    pass


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (or None)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise DIError("libdi ops take CUDA tensors (no CPU fallback)")
    if not t.is_contiguous():
        raise DIError("libdi ops take contiguous tensors")
    return t.data_ptr()


class DeviceView:
    """Zero-copy torch view of a libdi-owned device buffer (via __cuda_array_interface__)."""

    def __init__(self, p: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(p), False),
                                         "version": 3, "strides": None}


def view(p, shape, dtype: str = "f32"):
    import torch
    ts = {"f32": "<f4", "f16": "<f2", "i32": "<i4"}[dtype]
    return torch.as_tensor(DeviceView(p if isinstance(p, int) else p.value, shape, ts), device="cuda")


def u32(*vals) -> ctypes.Array:
    return (ctypes.c_uint32 * len(vals))(*vals)


class Context:
    """One libdi context per device (the analogue of the WebGPU device the reference requests).

    Binds to torch's current CUDA stream so libdi launches order with torch's own work."""

    def __init__(self, device: int = 0, stream=None):
        import torch
        self.device = device
        h = ctypes.c_void_p()
        rc = lib().di_init(device, ctypes.byref(h))
        if rc != DI_OK:
            raise DIError(f"di_init({device}) failed with {rc}")
        self.h = h
        s = stream if stream is not None else torch.cuda.current_stream(device)
        self.stream = s
        self.check(lib().di_set_stream(self.h, ctypes.c_void_p(s.cuda_stream)), "di_set_stream")

    def check(self, rc: int, what: str = "libdi") -> None:
        if rc != DI_OK:
            msg = lib().di_last_error(self.h)
            raise DIError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")

    def fault(self) -> int:
        return lib().di_device_fault(self.h)

    def clear_fault(self) -> None:
        self.check(lib().di_clear_fault(self.h), "di_clear_fault")

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().di_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default = {}


def default_context(device: int = 0) -> Context:
    if device not in _default:
        _default[device] = Context(device)
    return _default[device]
