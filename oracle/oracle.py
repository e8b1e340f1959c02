"""ctypes front end of the CPU oracle (oracle/h3b_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, never by the product package.
Arrays are numpy; bf16 travels as uint16 bit patterns, e4m3 as uint8.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libh3b_oracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "h3b_oracle.c")
        ):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.h3bo_expf.restype = ctypes.c_float
        _lib.h3bo_expf.argtypes = [ctypes.c_float]
        _lib.h3bo_tanhf.restype = ctypes.c_float
        _lib.h3bo_tanhf.argtypes = [ctypes.c_float]
        _lib.h3bo_f32_to_e4m3.restype = ctypes.c_uint8
        _lib.h3bo_f32_to_e4m3.argtypes = [ctypes.c_float]
        _lib.h3bo_e4m3_to_f32.restype = ctypes.c_float
        _lib.h3bo_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        _lib.h3bo_f32_to_bf16.restype = ctypes.c_uint16
        _lib.h3bo_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.h3bo_f32_to_f16.restype = ctypes.c_uint16
        _lib.h3bo_f32_to_f16.argtypes = [ctypes.c_float]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


I64 = ctypes.c_int64

# ----------------------------------------------------------------------------- bf16 helpers


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    table = np.array([lib().h3bo_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return table[np.asarray(b, dtype=np.uint8)]


# ----------------------------------------------------------------------------- quantization


def quant_rowwise(x_bf16: np.ndarray):
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    lib().h3bo_quant_rowwise(_p(x), I64(M), I64(K), _p(q), _p(s))
    return q, s


def quant_rowwise_convrot(x_bf16: np.ndarray, act: int = 0):
    x = _c(x_bf16, np.uint16)
    M, W = x.shape
    K = W // 2 if act == 2 else W
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    lib().h3bo_quant_rowwise_convrot(_p(x), I64(M), I64(K), ctypes.c_int(act), _p(q), _p(s))
    return q, s


def fht256(v: np.ndarray) -> np.ndarray:
    out = np.array(v, dtype=np.float32, copy=True).reshape(-1, 256)
    for row in out:
        lib().h3bo_fht256(_p(row))
    return out.reshape(np.shape(v))


def rms_adaln_rows(x_bf16, w_bf16, scale_tab_bf16, shift_tab_bf16, seg_row=None, eps=1e-5):
    """The modulated rows the fused quantizer rotates and quantizes (bf16 values as float32)."""
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    w = _c(w_bf16, np.uint16)
    sc = _c(np.atleast_2d(scale_tab_bf16), np.uint16)
    sh = _c(np.atleast_2d(shift_tab_bf16), np.uint16)
    out = np.empty((M, K), np.float32)
    for m in range(M):
        r = 0 if seg_row is None else int(seg_row[m])
        lib().h3bo_rms_adaln_row(_p(x[m]), I64(K), _p(w), _p(sc[r]), _p(sh[r]), ctypes.c_float(eps), _p(out[m]))
    return out


def rms_adaln_quant(x_bf16, w_bf16, scale_tab_bf16, shift_tab_bf16, seg_row=None, eps=1e-5,
                    convrot=True):
    x = _c(x_bf16, np.uint16)
    M, K = x.shape
    w = _c(w_bf16, np.uint16)
    sc = _c(np.atleast_2d(scale_tab_bf16), np.uint16)
    sh = _c(np.atleast_2d(shift_tab_bf16), np.uint16)
    sr = _c(seg_row, np.int32)
    q = np.empty((M, K), np.int8)
    s = np.empty((M,), np.float32)
    lib().h3bo_rms_adaln_quant(_p(x), I64(M), I64(K), _p(w), _p(sc), _p(sh), _p(sr),
                               ctypes.c_float(eps), ctypes.c_int(int(convrot)),
                               _p(q), _p(s))
    return q, s


# ----------------------------------------------------------------------------- W4A8


def w4_decode(qdata: np.ndarray, s_rel: np.ndarray, codebook, group_size: int) -> np.ndarray:
    qd = _c(qdata, np.int8)
    N, Kh = qd.shape
    K = Kh * 2
    if s_rel.dtype == np.uint8:
        kind, sr = 1, _c(s_rel, np.uint8)
    else:
        kind, sr = 0, _c(s_rel, np.float32)
    cb = _c(codebook, np.float32)
    out = np.empty((N, K), np.int8)
    lib().h3bo_w4_decode(_p(qd), _p(sr), ctypes.c_int(kind), _p(cb), I64(N), I64(K), I64(group_size), _p(out))
    return out


# ----------------------------------------------------------------------------- GEMM


def gemm_i8(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = _c(a, np.int8)
    b = _c(b, np.int8)
    M, K = a.shape
    N = b.shape[0]
    acc = np.empty((M, N), np.int32)
    lib().h3bo_gemm_i8(_p(a), _p(b), I64(M), I64(N), I64(K), _p(acc))
    return acc


def epilogue(acc, xs, ws, bias=None, residual=None, gate=None):
    acc = _c(acc, np.int32)
    M, N = acc.shape
    xs = _c(xs, np.float32).reshape(-1)
    ws = _c(ws, np.float32).reshape(-1)
    b = None if bias is None else _c(bias, np.float32)
    if residual is not None:
        res = np.array(residual, dtype=np.uint16, copy=True)
        g = _c(gate, np.uint16)
        lib().h3bo_epilogue(_p(acc), I64(M), I64(N), _p(xs), _p(ws), I64(ws.size), _p(b), None,
                            _p(res), _p(g), I64(N))
        return res
    out = np.empty((M, N), np.uint16)
    lib().h3bo_epilogue(_p(acc), I64(M), I64(N), _p(xs), _p(ws), I64(ws.size), _p(b), _p(out),
                        None, None, I64(N))
    return out


def int8_linear(x_bf16, qweight, wscale, bias_f32=None, convrot=0, act=0, residual=None, gate=None):
    """Quantize + GEMM + epilogue, exactly as the CUDA library computes it."""
    if convrot:
        q, s = quant_rowwise_convrot(x_bf16, act)
    else:
        q, s = quant_rowwise(x_bf16)
    acc = gemm_i8(q, qweight)
    return epilogue(acc, s, wscale, bias_f32, residual, gate)


# ----------------------------------------------------------------------------- attention prep


def key_mean(k_bf16: np.ndarray) -> np.ndarray:
    k = _c(k_bf16, np.uint16)
    L, H, D = k.shape
    out = np.empty((H, D), np.uint16)
    lib().h3bo_key_mean(_p(k), I64(L), I64(H), I64(D), _p(out))
    return out


def pool_sim_quant(x_bf16, block: int, thr, mean=None):
    x = _c(x_bf16, np.uint16)
    L, H, D = x.shape
    nb = (L + block - 1) // block
    thr = _c(thr, np.float32)
    pooled = np.empty((H, nb, D), np.uint16)
    sim = np.empty((H, nb), np.uint8)
    q = np.empty((H, nb * block, D), np.int8)
    sc = np.empty((H, nb), np.float32)
    lib().h3bo_pool_sim_quant(_p(x), I64(L), I64(H), _p(_c(mean, np.uint16)), ctypes.c_int(block), _p(thr),
                              _p(pooled), _p(sim), _p(q), _p(sc))
    return pooled, sim, q, sc


def qk_rmsnorm_rope(qkv_bf16, H, q_off, k_off, qw, kw, cos_t, sin_t, rot=128, eps=1e-6):
    x = np.array(qkv_bf16, dtype=np.uint16, copy=True)
    L, stride = x.shape
    lib().h3bo_qk_rmsnorm_rope(_p(x), I64(L), I64(H), I64(stride), I64(q_off), I64(k_off),
                               _p(_c(qw, np.uint16)), _p(_c(kw, np.uint16)), _p(_c(cos_t, np.uint16)),
                               _p(_c(sin_t, np.uint16)), ctypes.c_int(rot), ctypes.c_float(eps))
    return x


def value_fp8(v_bf16, Lpad=None):
    v = _c(v_bf16, np.uint16)
    L, H, D = v.shape
    if Lpad is None:
        Lpad = (L + 127) // 128 * 128
    vt = np.empty((H, D, Lpad), np.uint8)
    vs = np.empty((H, D), np.float32)
    lib().h3bo_value_fp8(_p(v), I64(L), I64(H), I64(Lpad), _p(vt), _p(vs))
    return vt, vs


def block_mask(pooled_q, simq, pooled_k, simk, *, mode, budget, protected_kb=0, flags=0,
               temporal_radius=-1, temporal_spatial_radius=0, frames=0, frame_tokens=0,
               protected_tokens=0, q_tokens=0, q_index=None, protected_qb=0):
    pq = _c(pooled_q, np.uint16)
    pk = _c(pooled_k, np.uint16)
    H, Qb, _ = pq.shape
    Kb = pk.shape[1]
    words = (Kb + 31) // 32
    bm = np.zeros((H, Qb, words), np.uint32)
    bud = _c(np.broadcast_to(np.asarray(budget, np.float32), (H,)), np.float32)
    lib().h3bo_block_mask(_p(pq), _p(_c(simq, np.uint8)), I64(Qb), _p(pk), _p(_c(simk, np.uint8)), I64(Kb),
                          I64(H), ctypes.c_int(mode), _p(bud), I64(protected_kb), ctypes.c_int(flags),
                          ctypes.c_int(temporal_radius), ctypes.c_int(temporal_spatial_radius), I64(frames),
                          I64(frame_tokens), I64(protected_tokens), I64(q_tokens), _p(_c(q_index, np.int64)),
                          I64(protected_qb), _p(bm))
    return bm


def bitmap_to_bool(bm: np.ndarray, Kb: int) -> np.ndarray:
    bits = np.unpackbits(bm.view(np.uint8), axis=-1, bitorder="little")
    return bits[..., :Kb].astype(bool)


def bitmap_to_lut(bm: np.ndarray, Kb: int):
    bm = _c(bm, np.uint32)
    rows = int(np.prod(bm.shape[:-1]))
    lut = np.empty(bm.shape[:-1] + (Kb,), np.int32)
    valid = np.empty(bm.shape[:-1], np.int32)
    lib().h3bo_bitmap_to_lut(_p(bm), I64(rows), I64(Kb), _p(lut), _p(valid))
    return lut, valid


def attention(q_i8, q_scale, qblk, Lq, k_i8, k_scale, Lk, vt, v_scale, bitmap=None, sm_scale=None):
    q = _c(q_i8, np.int8)
    k = _c(k_i8, np.int8)
    H, Lqpad, D = q.shape
    Lkpad = k.shape[1]
    out = np.empty((Lq, H, D), np.uint16)
    if sm_scale is None:
        sm_scale = 1.0 / np.sqrt(D)
    lib().h3bo_attention(_p(q), _p(_c(q_scale, np.float32)), ctypes.c_int(qblk), I64(Lq), I64(Lqpad), _p(k),
                         _p(_c(k_scale, np.float32)), I64(Lk), I64(Lkpad), _p(_c(vt, np.uint8)),
                         _p(_c(v_scale, np.float32)), I64(H), _p(_c(bitmap, np.uint32)),
                         ctypes.c_float(sm_scale), _p(out))
    return out


def attention_kernel(q_i8, q_scale, Lq, k_i8, k_scale, Lk, vt, v_scale, bitmap=None, sm_scale=None, *,
                     q_gran=0, q_block=128, k_gran=0):
    """Attention in the GPU kernel's own arithmetic (h3bo_attention_kernel): lazy
    running max, P = 2^x * 112 rounded to E4M3, fp32 row sums in the kernel's order.
    q_gran 0: q_block-row scale groups, 1: Sage per_thread; k_gran 0: per 64-key
    block, 1: Sage per_thread (4 groups per block)."""
    q = _c(q_i8, np.int8)
    k = _c(k_i8, np.int8)
    H, Lqpad, D = q.shape
    Lkpad = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / np.sqrt(D)
    if H > 1:
        # one call per head on a thread each (ctypes drops the GIL during the call)
        from concurrent.futures import ThreadPoolExecutor

        qs, ks, vsc = _c(q_scale, np.float32), _c(k_scale, np.float32), _c(v_scale, np.float32)
        bm = _c(bitmap, np.uint32)
        vt = _c(vt, np.uint8)

        def one(h):
            return attention_kernel(q[h:h + 1], qs[h:h + 1], Lq, k[h:h + 1], ks[h:h + 1], Lk, vt[h:h + 1],
                                    vsc[h:h + 1], None if bm is None else bm[h:h + 1], sm_scale, q_gran=q_gran,
                                    q_block=q_block, k_gran=k_gran)

        with ThreadPoolExecutor(max_workers=min(H, os.cpu_count() or 1)) as ex:
            return np.concatenate(list(ex.map(one, range(H))), axis=1)
    out = np.empty((Lq, H, D), np.uint16)
    lib().h3bo_attention_kernel(_p(q), _p(_c(q_scale, np.float32)), ctypes.c_int(q_gran), ctypes.c_int(q_block),
                                I64(Lq), I64(Lqpad), _p(k), _p(_c(k_scale, np.float32)), ctypes.c_int(k_gran),
                                I64(Lk), I64(Lkpad), _p(_c(vt, np.uint8)), _p(_c(v_scale, np.float32)), I64(H),
                                _p(_c(bitmap, np.uint32)), ctypes.c_float(sm_scale), _p(out))
    return out


def quant_per_thread(x_bf16, kind: int, mean=None):
    """Sage per_thread INT8 (h3bo_quant_per_thread): kind 0 Q (128-row blocks, 32
    groups), kind 1 K (64-row blocks, 4 groups, values bf16(k - mean))."""
    x = _c(x_bf16, np.uint16)
    L, H, D = x.shape
    blk, ng = (128, 32) if kind == 0 else (64, 4)
    nb = (L + blk - 1) // blk
    Lpad = (L + 127) // 128 * 128
    q = np.empty((H, Lpad, D), np.int8)
    q[:, nb * blk:] = 0
    sc = np.empty((H, nb * ng), np.float32)
    lib().h3bo_quant_per_thread(_p(x), I64(L), I64(H), _p(_c(mean, np.uint16)), ctypes.c_int(kind), _p(q),
                                I64(Lpad), _p(sc))
    return q, sc


def w4a8_correction(xq, xs, G: int, corr_bf16, out_bf16):
    """The W4A8 group correction added into out (h3bo_w4a8_correction); returns new bits."""
    xq = _c(xq, np.int8)
    M, K = xq.shape
    corr = _c(corr_bf16, np.uint16)
    N = corr.shape[1]
    out = np.array(out_bf16, dtype=np.uint16, copy=True)
    lib().h3bo_w4a8_correction(_p(xq), _p(_c(xs, np.float32).reshape(-1)), I64(M), I64(K), I64(G), _p(corr), I64(N),
                               _p(out))
    return out
