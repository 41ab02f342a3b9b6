"""ctypes front end of the CPU oracle (``oracle/moe_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline legs as the checker.  The product library never
imports it.

All bf16 tensors are numpy ``uint16`` arrays holding the raw bf16 bits.  The
functions restate (file:line within the reference project):

* ``route_topk``      aptransformer/ESRouter.mm:14-32
* ``route_weights``   aptransformer/ESRouter.mm:34-40
* ``experts_sparse``  aptransformer/ESExperts.mm:44-60 (gather_mm path)
* ``experts_sparse_q`` aptransformer/ESExperts.mm:44-60 (gather_qmm path)
* ``experts_dense``   aptransformer/ESExperts.mm:28-42
* ``gelu_tanh_bf16``  aptransformer/ESOps.h:29-37
* ``quantize_affine`` mx::quantize (affine), called at ESExperts.mm:14,16
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "moe_oracle.c"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "libmoe_oracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, i64, f32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.oracle_route_topk.argtypes = [P, i32, i32, P, P, P, i32, i32, f32, P, P, P, P, P]
        L.oracle_route_weights.argtypes = [P, P, i32, i32, i32, P]
        L.oracle_experts_sparse.argtypes = [P, i32, i32, i32, i32, P, P, P, P, P, P]
        L.oracle_experts_sparse_q.argtypes = [P, i32, i32, i32, i32, P, P, P, P, P, P, i32, i32,
                                              P, P, P, P]
        L.oracle_experts_dense.argtypes = [P, i32, i32, i32, i32, P, P, P, P]
        L.oracle_gelu_tanh_bf16.argtypes = [P, P, i64]
        L.oracle_gelu_tanh_f32.argtypes = [f32]
        L.oracle_gelu_tanh_f32.restype = f32
        L.oracle_bf16_round.argtypes = [f32]
        L.oracle_bf16_round.restype = f32
        L.oracle_quantize_affine.argtypes = [P, i64, i32, i32, i32, P, P, P]
        L.oracle_quantize_affine.restype = i32
        L.oracle_dequantize_affine.argtypes = [P, P, P, i64, i32, i32, i32, P]
        L.oracle_rms_norm.argtypes = [P, P, i32, i32, f32, P]
        L.oracle_num_threads.restype = i32
        L.oracle_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- bf16 helpers

def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- router

def route_topk(x, proj, scale, pes, top_k, eps=1e-6, return_scores=False):
    x, proj, scale, pes = (_c(a, np.uint16) for a in (x, proj, scale, pes))
    T, H = x.shape
    E = proj.shape[0]
    idx = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), np.uint16)
    scores = np.zeros((T, E), np.float32)
    probs = np.zeros((T, E), np.float32)
    wf = np.zeros((T, top_k), np.float32)
    lib().oracle_route_topk(_p(x), T, H, _p(proj), _p(scale), _p(pes), E, top_k, eps,
                            _p(idx), _p(w), _p(scores), _p(probs), _p(wf))
    if return_scores:
        return idx, w, dict(scores=scores, probs=probs, w_f32=wf)
    return idx, w


def route_weights(idx, w, num_experts):
    idx, w = _c(idx, np.int32), _c(w, np.uint16)
    T, K = idx.shape
    W = np.zeros((T, num_experts), np.uint16)
    lib().oracle_route_weights(_p(idx), _p(w), T, num_experts, K, _p(W))
    return W


# ---------------------------------------------------------------- experts

def experts_sparse(x, gate_up, down, idx, w, return_pairs=False):
    x, gate_up, down = (_c(a, np.uint16) for a in (x, gate_up, down))
    idx, w = _c(idx, np.int32), _c(w, np.uint16)
    T, H = x.shape
    K = idx.shape[1]
    I = down.shape[2]
    out = np.zeros((T, H), np.uint16)
    pairs = np.zeros((T * K, H), np.uint16) if return_pairs else None
    lib().oracle_experts_sparse(_p(x), T, H, I, K, _p(gate_up), _p(down), _p(idx), _p(w),
                                _p(out), _p(pairs))
    return (out, pairs) if return_pairs else out


def experts_sparse_q(x, gu_q, gu_s, gu_b, dn_q, dn_s, dn_b, bits, group_size, idx, w, inter):
    x = _c(x, np.uint16)
    gu_q, dn_q = _c(gu_q, np.uint32), _c(dn_q, np.uint32)
    gu_s, gu_b, dn_s, dn_b = (_c(a, np.uint16) for a in (gu_s, gu_b, dn_s, dn_b))
    idx, w = _c(idx, np.int32), _c(w, np.uint16)
    T, H = x.shape
    K = idx.shape[1]
    out = np.zeros((T, H), np.uint16)
    lib().oracle_experts_sparse_q(_p(x), T, H, inter, K, _p(gu_q), _p(gu_s), _p(gu_b),
                                  _p(dn_q), _p(dn_s), _p(dn_b), bits, group_size,
                                  _p(idx), _p(w), _p(out), None)
    return out


def experts_dense(x, gate_up, down, W):
    x, gate_up, down, W = (_c(a, np.uint16) for a in (x, gate_up, down, W))
    T, H = x.shape
    E = gate_up.shape[0]
    I = down.shape[2]
    out = np.zeros((T, H), np.uint16)
    lib().oracle_experts_dense(_p(x), T, H, I, E, _p(gate_up), _p(down), _p(W), _p(out))
    return out


def gelu_tanh_bf16(x):
    x = _c(x, np.uint16)
    y = np.zeros_like(x)
    lib().oracle_gelu_tanh_bf16(_p(x), _p(y), x.size)
    return y


def gelu_tanh_f32(v: float) -> float:
    return lib().oracle_gelu_tanh_f32(v)


# ---------------------------------------------------------------- quantisation

def quantize_affine(w, group_size=64, bits=4):
    """w [..., cols] bf16 -> (q u32 [..., cols*bits/32], scales, biases [..., cols/gs] bf16)."""
    w = _c(w, np.uint16)
    lead, cols = w.shape[:-1], w.shape[-1]
    rows = int(np.prod(lead)) if lead else 1
    q = np.zeros(lead + (cols * bits // 32,), np.uint32)
    s = np.zeros(lead + (cols // group_size,), np.uint16)
    b = np.zeros_like(s)
    rc = lib().oracle_quantize_affine(_p(w), rows, cols, group_size, bits, _p(q), _p(s), _p(b))
    if rc:
        raise ValueError(f"unsupported quantisation bits={bits} gs={group_size} cols={cols}")
    return q, s, b


def dequantize_affine(q, s, b, group_size=64, bits=4):
    q = _c(q, np.uint32)
    s, b = _c(s, np.uint16), _c(b, np.uint16)
    cols = q.shape[-1] * 32 // bits
    rows = int(np.prod(q.shape[:-1])) if q.ndim > 1 else 1
    out = np.zeros(q.shape[:-1] + (cols,), np.float32)
    lib().oracle_dequantize_affine(_p(q), _p(s), _p(b), rows, cols, group_size, bits, _p(out))
    return out


def rms_norm(x, weight=None, eps=1e-6):
    """ESRMSNorm::forward (ESRMSNorm.mm:14-28): f32 inside, bf16 out."""
    x = _c(x, np.uint16)
    T, H = x.shape
    out = np.zeros_like(x)
    wt = None if weight is None else _c(weight, np.uint16)
    lib().oracle_rms_norm(_p(x), _p(wt), T, H, eps, _p(out))
    return out


def layer_moe(x1, pre_w, post_w, proj, scale, pes, gate_up, down, top_k, eps=1e-6):
    """The MoE part of ESDecoderLayer::forward (ESDecoderLayer.mm:69-74):
    post_ff_ln_2(experts(pre_ff_ln_2(x1), router(x1)))."""
    exp_in = rms_norm(x1, pre_w, eps)
    idx, w = route_topk(x1, proj, scale, pes, top_k, eps)
    moe = experts_sparse(exp_in, gate_up, down, idx, w)
    return rms_norm(moe, post_w, eps), idx, w


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(n)


def bf16_add(a, b) -> np.ndarray:
    """bf16 + bf16 -> bf16 (f32 add, one rounding), as mx::add on bf16 arrays."""
    return f32_to_bf16(bf16_to_f32(a) + bf16_to_f32(b))


def decoder_ff(x1, hmlp, pre_w, ln1_w, post_w, ff_w, proj, scale, pes, gate_up, down, top_k,
               eps=1e-6):
    """Feed-forward tail of an MoE decoder layer (ESDecoderLayer.mm:61-78) given
    the dense MLP output hmlp: x2 = x1 + post_ff_ln(post_ff_ln_1(hmlp) +
    post_ff_ln_2(MoE(x1)))."""
    moe, idx, w = layer_moe(x1, pre_w, post_w, proj, scale, pes, gate_up, down, top_k, eps)
    dense = rms_norm(hmlp, ln1_w, eps)
    ff = bf16_add(dense, moe)
    return bf16_add(x1, rms_norm(ff, ff_w, eps)), idx, w


def mlp(x, gate, up, down):
    """ESMLPBlock::forward (ESMLPBlock.mm:11-15): down(bf16(gelu(bf16 gate(x))) *
    bf16 up(x)) -- the expert arithmetic with one expert of weight 1."""
    gu = np.concatenate([_c(gate, np.uint16), _c(up, np.uint16)], 0)[None]
    dn = _c(down, np.uint16)[None]
    T = np.asarray(x).shape[0]
    idx = np.zeros((T, 1), np.int32)
    w = f32_to_bf16(np.ones((T, 1), np.float32))
    return experts_sparse(x, gu, dn, idx, w)


def decoder_ff_full(x1, pre_ff_w, gate, up, down, pre_w, ln1_w, post_w, ff_w, proj, scale, pes,
                    gate_up, down_e, top_k, eps=1e-6):
    """ESDecoderLayer.mm:61-78 from x1: the dense MLP on pre_ff_ln(x1) plus the
    MoE, with the trailing norms and the residual add."""
    hmlp = mlp(rms_norm(x1, pre_ff_w, eps), gate, up, down)
    return decoder_ff(x1, hmlp, pre_w, ln1_w, post_w, ff_w, proj, scale, pes, gate_up, down_e,
                      top_k, eps)

