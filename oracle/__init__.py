"""CPU oracle (TEST INFRASTRUCTURE ONLY): numpy wrappers over oracle/_build/liboracle.so.

The C++ restatement of the reference's WGSL / JS math lives in oracle.cpp (each function cites the
reference file:line it follows).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
use this module, and only as the checker or the timed CPU baseline — never on the product path.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "liboracle.so"

_lib = None
_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32 = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_i32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_I, _U64, _SZ, _F, _C = ctypes.c_int, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_float, ctypes.c_char_p

_SIGS = {
    "o_gen_uniform": [_U64, _C, _SZ, _F, _f],
    "o_gen_normal": [_U64, _C, _SZ, _F, _F, _f],
    "o_f16_to_f32": [_u16, _f, _SZ],
    "o_f32_to_f16": [_f, _u16, _SZ],
    "o_sched_timesteps": [_I, _f],
    "o_sched_sigmas": [_I, _f],
    "o_sched_scale_input": [_f, _f, _SZ, _F],
    "o_sched_step": [_f, _f, _f, _SZ, _F, _F],
    "o_noise_latent": [_I, _I, _I, _I, _F, _f],
    "o_unary": [_I, _f, _f, _SZ],
    "o_binary": [_I, _f, _SZ, _f, _SZ, _f, _SZ],
    "o_binary_bcast": [_I, _f, _f, _f, _u32],
    "o_affine_bcast": [_f, _f, _f, _f, _u32],
    "o_softmax": [_f, _f, ctypes.c_uint32, ctypes.c_uint32],
    "o_instance_norm": [_f, _f, _f, _f, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32],
    "o_group_norm": [_f, _f, _f, _f, _I, _I, _I, _I, _F, _I, _I],
    "o_layer_norm": [_f, _f, _f, _f, _I, _I, _F],
    "o_matmul": [_f, _f, _f, _I, _I, _I, _I, _I],
    "o_gemm": [_f, _f, _f, _f, _I, _I, _I, _I],
    "o_conv": [_f, _f, _f, _f, _I, _I, _I, _I, _I, _I, _I, _I],
    "o_resize_nearest": [_f, _f, _u32],
    "o_reduce_mean": [_f, _f, ctypes.c_uint32, ctypes.c_uint32],
    "o_transpose": [_f, _f, _u32],
    "o_pow_scalar": [_f, _f, _SZ, _F],
    "o_slice": [_f, _f, _u32],
    "o_concat_copy": [_f, _f, _u32],
    "o_attention": [_f, _f, _f, _f, _I, _I, _I, _I, _I, ctypes.c_void_p, _I],
    "o_tembed": [_f, _I, _f, _f, _f, _f, _I, _I, _f],
    "o_resnet_block": [_f, _f, _I, _I, _I, _I, _I, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _F, _I, _f],
    "o_transformer_block": [_f, _f, _I, _I, _I, _I, _I, _U64, _I, _f],
    "o_unet_forward": [_f, _f, _f, _I, _I, _I, _I, _U64, _f],
    "o_vae_decode": [_f, _I, _I, _I, _U64, _f],
    "o_attention_causal": [_f, _f, _f, _f, _I, _I, _I, _I],
    "o_text_encode": [_i32, _I, _I, _I, _U64, _f],
    "o_num_threads": [],
    "o_set_threads": [_I],
    "o_param_seconds": [],
    "o_clear_cache": [],
}
_RES = {"o_num_threads": ctypes.c_int, "o_param_seconds": ctypes.c_double}


def build() -> Path:
    """Compiles liboracle.so with the committed Makefile (system g++ with OpenMP)."""
    src = ORACLE_DIR / "oracle.cpp"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        for n, a in _SIGS.items():
            fn = getattr(L, n)
            fn.argtypes = a
            fn.restype = _RES.get(n)
        _lib = L
    return _lib


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


# ---- generator / conversions ----
def gen_uniform(seed: int, name: str, n: int, bound: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().o_gen_uniform(seed, name.encode(), n, bound, out)
    return out


def gen_normal(seed: int, name: str, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().o_gen_normal(seed, name.encode(), n, mean, std, out)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = _c(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().o_f16_to_f32(h.ravel(), out.ravel(), h.size)
    return out


def f32_to_f16(f: np.ndarray) -> np.ndarray:
    f = _c(f)
    out = np.empty(f.shape, np.uint16)
    lib().o_f32_to_f16(f.ravel(), out.ravel(), f.size)
    return out


# ---- scheduler ----
def sched_timesteps(n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().o_sched_timesteps(n, out)
    return out


def sched_sigmas(n: int) -> np.ndarray:
    out = np.empty(n + 1, np.float32)
    lib().o_sched_sigmas(n, out)
    return out


def sched_scale_input(x, sigma: float) -> np.ndarray:
    """scaleModelInput (scheduler.js:95-101): float(double(x) / sqrt(sigma^2 + 1))."""
    x = _c(x)
    y = np.empty_like(x)
    lib().o_sched_scale_input(x.ravel(), y.ravel(), x.size, sigma)
    return y


def sched_step(x, eps, sig_i: float, sig_next: float) -> np.ndarray:
    """Euler step (scheduler.js:105-110): float(double(x) + (sig_next - sig_i) * double(eps))."""
    x = _c(x)
    y = np.empty_like(x)
    lib().o_sched_step(x.ravel(), _c(eps).ravel(), y.ravel(), x.size, sig_i, sig_next)
    return y


def noise_latent(B: int, H: int, W: int, seed: int, sigma: float) -> np.ndarray:
    out = np.empty(B * 4 * H * W, np.float32)
    lib().o_noise_latent(B, H, W, seed, sigma, out)
    return out.reshape(B, 4, H, W)


# ---- op families ----
def unary(op: int, x):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_unary(op, x.ravel(), y.ravel(), x.size)
    return y


def binary(op: int, a, b, n=None):
    a, b = _c(a), _c(b)
    n = n or max(a.size, b.size)
    y = np.empty(n, np.float32)
    lib().o_binary(op, a.ravel(), a.size, b.ravel(), b.size, y, n)
    return y


def binary_bcast(op, a, b, cfg):
    cfg = _c(cfg, np.uint32)
    y = np.empty(int(cfg[16]), np.float32)
    lib().o_binary_bcast(op, _c(a).ravel(), _c(b).ravel(), y, cfg)
    return y


def affine_bcast(a, g, b, cfg):
    cfg = _c(cfg, np.uint32)
    y = np.empty(int(cfg[16]), np.float32)
    lib().o_affine_bcast(_c(a).ravel(), _c(g).ravel(), _c(b).ravel(), y, cfg)
    return y


def softmax(x, inner, rows):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_softmax(x.ravel(), y.ravel(), inner, rows)
    return y


def instance_norm(x, g, b, C, HW, N):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_instance_norm(x.ravel(), _c(g), _c(b), y.ravel(), C, HW, N)
    return y


def group_norm(x, g, b, N, C, HW, G, eps, silu=False, clamp=True):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_group_norm(x.ravel(), _c(g), _c(b), y.ravel(), N, C, HW, G, eps, int(silu), int(clamp))
    return y


def layer_norm(x, g, b, rows, D, eps=1e-5):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_layer_norm(x.ravel(), _c(g), _c(b), y.ravel(), rows, D, eps)
    return y


def matmul(A, B, M, N, K, b_batched, batch):
    y = np.empty(batch * M * N, np.float32)
    lib().o_matmul(_c(A).ravel(), _c(B).ravel(), y, M, N, K, b_batched, batch)
    return y


def gemm(A, B, C, M, N, K, transB):
    y = np.empty(M * N, np.float32)
    lib().o_gemm(_c(A).ravel(), _c(B).ravel(), _c(C).ravel(), y, M, N, K, transB)
    return y


def conv(x, w, b, N, Ci, H, W, Co, K, S, PAD):
    Ho, Wo = (H + 2 * PAD - K) // S + 1, (W + 2 * PAD - K) // S + 1
    y = np.empty(N * Co * Ho * Wo, np.float32)
    lib().o_conv(_c(x).ravel(), _c(w).ravel(), _c(b).ravel(), y, N, Ci, H, W, Co, K, S, PAD)
    return y.reshape(N, Co, Ho, Wo)


def resize_nearest(x, cfg):
    cfg = _c(cfg, np.uint32)
    y = np.empty(int(cfg[5]), np.float32)
    lib().o_resize_nearest(_c(x).ravel(), y, cfg)
    return y


def reduce_mean(x, inner, rows):
    y = np.empty(rows, np.float32)
    lib().o_reduce_mean(_c(x).ravel(), y, inner, rows)
    return y


def transpose(x, cfg):
    cfg = _c(cfg, np.uint32)
    y = np.empty(int(cfg[16]), np.float32)
    lib().o_transpose(_c(x).ravel(), y, cfg)
    return y


def pow_scalar(x, e):
    x = _c(x)
    y = np.empty_like(x)
    lib().o_pow_scalar(x.ravel(), y.ravel(), x.size, e)
    return y


def slice_(x, cfg):
    cfg = _c(cfg, np.uint32)
    y = np.empty(int(cfg[16]), np.float32)
    lib().o_slice(_c(x).ravel(), y, cfg)
    return y


def concat_copy(x, y_init, cfg):
    y = _c(y_init).copy()
    lib().o_concat_copy(_c(x).ravel(), y.ravel(), _c(cfg, np.uint32))
    return y


# ---- fused blocks ----
def attention(q, k, v, B, H, Sq, Skv, layout=0, rows=None):
    """softmax(q k^T / 8) v, head dim 64; rows (optional) restricts the query rows computed."""
    q, k, v = _c(q), _c(k), _c(v)
    o = np.zeros(q.shape, np.float32)
    if rows is not None:
        r = _c(rows, np.int32)
        lib().o_attention(q.ravel(), k.ravel(), v.ravel(), o.ravel(), B, H, Sq, Skv, layout,
                          r.ctypes.data_as(ctypes.c_void_p), r.size)
    else:
        lib().o_attention(q.ravel(), k.ravel(), v.ravel(), o.ravel(), B, H, Sq, Skv, layout, None, 0)
    return o


def tembed(t, W1, b1, W2, b2, Din, Dh):
    t = _c(np.atleast_1d(t))
    y = np.empty(t.size * Dh, np.float32)
    lib().o_tembed(t, t.size, _c(W1).ravel(), _c(b1), _c(W2).ravel(), _c(b2), Din, Dh, y)
    return y.reshape(t.size, Dh)


def resnet_block(x, temb, g1, be1, w1, bb1, wt, bt, g2, be2, w2, bb2, eps=1e-5, temb_silu=True):
    N, C, H, W = x.shape
    y = np.empty_like(_c(x))
    lib().o_resnet_block(_c(x).ravel(), _c(temb).ravel(), N, C, H, W, temb.shape[-1], _c(g1), _c(be1),
                         _c(w1).ravel(), _c(bb1), _c(wt).ravel(), _c(bt), _c(g2), _c(be2), _c(w2).ravel(), _c(bb2),
                         eps, int(temb_silu), y.ravel())
    return y


def transformer_block(hidden, ctx, seed, fp16_weights=True):
    B, S, C = hidden.shape
    _, Sk, Cc = ctx.shape
    out = np.empty_like(_c(hidden))
    lib().o_transformer_block(_c(hidden).ravel(), _c(ctx).ravel(), B, S, C, Sk, Cc, seed, int(fp16_weights),
                              out.ravel())
    return out


def unet_forward(latent, t, ctx, seed):
    B, _, H, W = latent.shape
    Sk = ctx.shape[1]
    out = np.empty_like(_c(latent))
    tv = _c(np.broadcast_to(np.asarray(t, np.float32), (B,)))
    lib().o_unet_forward(_c(latent).ravel(), tv, _c(ctx).ravel(), B, H, W, Sk, seed, out.ravel())
    return out


def vae_decode(latent, seed):
    """SD VAE decoder on [B, 4, h, w] latents -> [B, 3, 8h, 8w] (latent / 0.18215 applied first)."""
    B, _, h, w = latent.shape
    out = np.empty((B, 3, 8 * h, 8 * w), np.float32)
    lib().o_vae_decode(_c(latent).ravel(), B, h, w, seed, out.ravel())
    return out


def attention_causal(q, k, v, layout=0):
    """Causal attention, head dim 64: query i sees keys 0..i.  layout 0 [B,S,H,64], 1 [B,H,S,64]."""
    if layout == 0:
        B, S, H, _ = q.shape
    else:
        B, H, S, _ = q.shape
    o = np.empty_like(_c(q))
    lib().o_attention_causal(_c(q).ravel(), _c(k).ravel(), _c(v).ravel(), o.ravel(), B, H, S, layout)
    return o


def text_encode(ids, layers, seed):
    """OpenCLIP ViT-H text encoder on int32 ids [B, S] -> [B, S, 1024] (final LayerNorm applied)."""
    ids = np.ascontiguousarray(ids, np.int32)
    B, S = ids.shape
    out = np.empty((B, S, 1024), np.float32)
    lib().o_text_encode(ids.ravel(), B, S, layers, seed, out.ravel())
    return out


def num_threads() -> int:
    return lib().o_num_threads()


def set_threads(n: int) -> None:
    lib().o_set_threads(int(n))


def param_seconds() -> float:
    """Cumulative seconds spent drawing parameters (the U-Net keeps them cached per seed)."""
    return lib().o_param_seconds()


def clear_cache() -> None:
    lib().o_clear_cache()
