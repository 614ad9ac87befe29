"""CPU restatement of the reference Gated DeltaNet recurrence (numpy).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against; it is never the thing measured or shipped.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.

Parity pin: the functions below restate, operation by operation, the two
Triton kernels of the reference solution and are checked against golden
vectors produced by running those kernels (``tests/golden/make_golden.py``):

* ``gates``    follows ``solution/triton/kernel_decode.py:46-55`` (decode) and
               ``solution/triton/kernel_prefill.py:108-113`` (prefill):
               ``x = a + dt_bias``; ``softplus(x) = x if x > 20 else log(1 + e^x)``;
               ``g = exp(-exp(A_log) * softplus(x))``; ``beta = sigmoid(b)``.
* ``decode``   follows ``kernel_decode.py:57-103`` and the host wrapper
               ``kernel_decode.py:115-183`` (default scale ``1/sqrt(d)`` when the
               scale is None or 0, zero state when the state is None, GVA head
               mapping ``qk_head = v_head // (HV // HQ)``).
* ``decode_pooled`` (multi-token decode against a state pool) follows
               ``_gdn_mtp_reference`` of the installed flashinfer (third party).
* ``prefill``  follows ``kernel_prefill.py:42-142`` and its host wrapper
               ``kernel_prefill.py:156-231``: a token-serial decode recurrence
               per (sequence, v-head); an empty sequence passes its initial
               state through unchanged (``kernel_prefill.py:65-73``).

Order of operations per state row v (k-last layout, row = one v index):
``S <- g*S``; ``u = S.k``; ``delta = beta*(v - u)``; ``S <- S + delta*k``;
``o = scale * S.q`` (output rounded to bf16, state kept in fp32).

The optional ``use_qk_l2norm`` flag has no counterpart in the reference (its
kernels never normalise q/k); it defines the library's optional fused
normalisation ``x * rsqrt(sum(x^2) + 1e-6)`` so the CUDA flag can be checked.

bf16 tensors are exchanged as ``uint16`` bit patterns (round-to-nearest-even).
"""

from __future__ import annotations

import math

import numpy as np

L2NORM_EPS = np.float32(1e-6)


# --------------------------------------------------------------------------
# bf16 <-> fp32 bit helpers
# --------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    out = rounded.astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> np.uint64(16)) | np.uint64(0x40)).astype(np.uint16)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def default_scale(scale, head_dim: int) -> np.float32:
    """``kernel_decode.py:124-125`` / ``kernel_prefill.py:166-167``: None or 0 -> 1/sqrt(d)."""
    if scale is None or float(scale) == 0.0:
        return np.float32(1.0 / math.sqrt(head_dim))
    return np.float32(scale)


# --------------------------------------------------------------------------
# gates
# --------------------------------------------------------------------------
def gates(A_log: np.ndarray, a: np.ndarray, dt_bias: np.ndarray, b: np.ndarray):
    """Decay g and write strength beta (``kernel_decode.py:52-55``).

    ``a`` and ``b`` are float32 (already widened from bf16) with the v-head
    axis last; ``A_log`` and ``dt_bias`` are float32 ``[HV]``.
    """
    with np.errstate(over="ignore"):
        x = (a + dt_bias).astype(np.float32)
        softplus = np.where(x > np.float32(20.0), x,
                            np.log(np.float32(1.0) + np.exp(x))).astype(np.float32)
        g = np.exp(-np.exp(A_log.astype(np.float32)) * softplus).astype(np.float32)
        beta = (np.float32(1.0) / (np.float32(1.0) + np.exp(-b))).astype(np.float32)
    return g, beta


def l2norm(x: np.ndarray) -> np.ndarray:
    """Optional q/k normalisation over the last axis (library extension)."""
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x / np.sqrt(ss + L2NORM_EPS)).astype(np.float32)


def _rows_step(S, kk, qq, vv, g, beta, scale):
    """One recurrence step on a block of states.

    S: [..., V, K] fp32; kk, qq: [..., K]; vv: [..., V]; g, beta: [...].
    Follows ``kernel_decode.py:83-87`` exactly in operation order.
    """
    S = g[..., None, None] * S
    old_v = np.einsum("...vk,...k->...v", S, kk, dtype=np.float32)
    delta = beta[..., None] * (vv - old_v)
    S = S + delta[..., :, None] * kk[..., None, :]
    out = scale * np.einsum("...vk,...k->...v", S, qq, dtype=np.float32)
    return S.astype(np.float32), out.astype(np.float32)


# --------------------------------------------------------------------------
# decode
# --------------------------------------------------------------------------
def decode(q, k, v, state, A_log, a, dt_bias, b, scale=None, use_qk_l2norm=False):
    """One-token GDN decode step (``kernel_decode.py:115-183``).

    q, k: uint16 bf16 bits ``[B, 1, HQ, D]``; v: ``[B, 1, HV, D]``;
    state: float32 ``[B, HV, D, D]`` (k-last) or None (zeros);
    A_log, dt_bias: float32 ``[HV]``; a, b: uint16 bf16 bits ``[B, 1, HV]``.
    Returns (out uint16 bf16 bits ``[B, 1, HV, D]``, new_state float32).
    """
    B, _, HQ, D = q.shape
    HV = v.shape[2]
    if HV % HQ != 0:
        raise ValueError("num_v_heads must be a multiple of num_q_heads")
    scale = default_scale(scale, D)
    qf = bf16_bits_to_f32(q)[:, 0]
    kf = bf16_bits_to_f32(k)[:, 0]
    vf = bf16_bits_to_f32(v)[:, 0]
    if use_qk_l2norm:
        qf, kf = l2norm(qf), l2norm(kf)
    ratio = HV // HQ
    qh = np.repeat(qf, ratio, axis=1)  # GVA: v-head h reads qk-head h // ratio
    kh = np.repeat(kf, ratio, axis=1)
    g, beta = gates(A_log, bf16_bits_to_f32(a)[:, 0], dt_bias, bf16_bits_to_f32(b)[:, 0])
    S = np.zeros((B, HV, D, D), np.float32) if state is None else np.asarray(state, np.float32)
    S, out = _rows_step(S, kh, qh, vf, g, beta, scale)
    return f32_to_bf16_bits(out)[:, None], S


# --------------------------------------------------------------------------
# prefill
# --------------------------------------------------------------------------
def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, use_qk_l2norm=False):
    """Variable-length GDN prefill (``kernel_prefill.py:156-231``).

    q, k: uint16 bf16 bits ``[T, HQ, D]``; v: ``[T, HV, D]``; a, b: ``[T, HV]``;
    state float32 ``[N, HV, D, D]`` or None; cu_seqlens integer ``[N+1]``.
    Returns (out uint16 bf16 bits ``[T, HV, D]``, new_state float32 ``[N, HV, D, D]``).
    Token-serial, exactly as ``kernel_prefill.py:88-134``.
    """
    T, HQ, D = q.shape
    HV = v.shape[1]
    cu = np.asarray(cu_seqlens).astype(np.int64)
    N = cu.shape[0] - 1
    scale = default_scale(scale, D)
    qf, kf, vf = bf16_bits_to_f32(q), bf16_bits_to_f32(k), bf16_bits_to_f32(v)
    if use_qk_l2norm:
        qf, kf = l2norm(qf), l2norm(kf)
    ratio = HV // HQ
    g, beta = gates(A_log, bf16_bits_to_f32(a), dt_bias, bf16_bits_to_f32(b))
    out = np.zeros((T, HV, D), np.float32)
    new_state = np.zeros((N, HV, D, D), np.float32)
    for n in range(N):
        S = np.zeros((HV, D, D), np.float32) if state is None else np.array(state[n], np.float32)
        for t in range(int(cu[n]), int(cu[n + 1])):
            qh = np.repeat(qf[t], ratio, axis=0)
            kh = np.repeat(kf[t], ratio, axis=0)
            S, out[t] = _rows_step(S, kh, qh, vf[t], g[t], beta[t], scale)
        new_state[n] = S  # empty sequence: initial state passes through (kernel_prefill.py:65-73)
    return f32_to_bf16_bits(out), new_state


# --------------------------------------------------------------------------
# pooled-state multi-token decode (serving form)
# --------------------------------------------------------------------------
def decode_pooled(q, k, v, pool, indices, A_log, a, dt_bias, b, scale=None, use_qk_l2norm=False,
                  return_intermediate=False):
    """Multi-token decode against a state pool (the serving form).

    Follows ``_gdn_mtp_reference`` of ``flashinfer/trace/templates/gdn.py``
    (flashinfer 0.6.11.post2, third party; the starter kit has no multi-token
    entry point): sequence i runs the token-serial recurrence of
    ``kernel_decode.py:83-87`` for T tokens from ``pool[indices[i]]``, writes every
    token's output and the final state back to that slot.  A negative index skips
    the sequence and leaves its outputs zero (the serving convention for padded
    entries; the third-party reference would index from the end of the pool).

    q, k ``[B, T, HQ, D]``, v ``[B, T, HV, D]``, a, b ``[B, T, HV]`` (bf16 bits);
    pool float32 ``[P, HV, D, D]``; indices int ``[B]``.
    Returns (out bf16 bits ``[B, T, HV, D]``, updated pool) and, with
    ``return_intermediate``, also ``{(slot, t): state after token t}``.
    """
    B, T, HQ, D = q.shape
    HV = v.shape[2]
    scale = default_scale(scale, D)
    ratio = HV // HQ
    pool = np.array(pool, np.float32, copy=True)
    out = np.zeros((B, T, HV, D), np.float32)
    inter = {}
    for i in range(B):
        slot = int(indices[i])
        if slot < 0:
            continue
        qf, kf, vf = bf16_bits_to_f32(q[i]), bf16_bits_to_f32(k[i]), bf16_bits_to_f32(v[i])
        if use_qk_l2norm:
            qf, kf = l2norm(qf), l2norm(kf)
        g, beta = gates(A_log, bf16_bits_to_f32(a[i]), dt_bias, bf16_bits_to_f32(b[i]))
        S = np.array(pool[slot], np.float32)
        for t in range(T):
            qh = np.repeat(qf[t], ratio, axis=0)
            kh = np.repeat(kf[t], ratio, axis=0)
            S, out[i, t] = _rows_step(S, kh, qh, vf[t], g[t], beta[t], scale)
            if return_intermediate:
                inter[(slot, t)] = S
        pool[slot] = S
    outb = f32_to_bf16_bits(out)
    outb[np.asarray(indices) < 0] = 0
    if return_intermediate:
        return outb, pool, inter
    return outb, pool
