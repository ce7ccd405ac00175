"""Device-resident compositions of the NPL benchmark workloads, as one caller
of the nplk_* ABI runs them back to back on one stream. The benchmark times
these functions and the parity tests check the same functions' outputs
against the reference's own CPU chain, so what is timed is what is checked.

All tensors are contiguous fp32 CUDA tensors on the current device; `stream`
is a cudaStream_t as c_void_p. Each function returns 0 or the first non-zero
library return code.
"""
from __future__ import annotations

import ctypes as C


def _p(t):
    return C.c_void_p(t.data_ptr())


def bandwidth_chain(lib, stream, x, w, mean, var, gamma, beta, dw_out, act_out, gap, probs,
                    eps: float = 1e-5) -> int:
    """depthwise 3x3 (stride 1, pad 1, no bias) -> inference batch norm ->
    ReLU in place -> global average pool -> softmax over the channels of each
    image: the reference's npl_depthwise_conv2d (npl_convolution.cpp:60-90),
    npl_batch_norm (npl_activation_norm.cpp:118-153), npl_relu (:51-54),
    npl_global_avg_pool (npl_pooling.cpp:63-87) and npl_softmax axis 1
    (npl_activation_norm.cpp:88-112).

    x, dw_out, act_out: [N, C, H, W]; w: [C, 1, 3, 3]; mean/var/gamma/beta:
    [C]; gap, probs: [N, C]. dw_out keeps the depthwise output, act_out the
    ReLU(BN(.)) output."""
    from . import conv_geom

    n, c, h, wd = x.shape
    g = conv_geom(n, c, h, wd, c, 3, 3, 1, 1)
    hw = h * wd
    rcs = (lib.nplk_depthwise_conv2d(stream, C.byref(g), _p(x), _p(w), None, _p(dw_out)),
           lib.nplk_batch_norm_infer(stream, n, c, hw, _p(dw_out), _p(act_out), _p(mean),
                                     _p(var), _p(gamma), _p(beta), eps),
           lib.nplk_activation(stream, n * c * hw, _p(act_out), _p(act_out), 1, 0.0, 0),
           lib.nplk_global_avg_pool(stream, n * c, hw, _p(act_out), _p(gap)),
           lib.nplk_softmax(stream, n, c, 1, _p(gap), _p(probs)))
    return next((r for r in rcs if r != 0), 0)


def bandwidth_chain_fused(lib, stream, x, w, mean, var, gamma, beta, gap, probs,
                          act_out=None, eps: float = 1e-5) -> int:
    """The same chain with its first four calls in one pass
    (nplk_depthwise_bn_act_gap: depthwise, BN, ReLU and the average pool
    without writing the intermediate maps; act_out, when given, receives the
    ReLU(BN(.)) map), then the softmax over the channels. gap and probs equal
    bandwidth_chain's bit for bit."""
    from . import conv_geom

    n, c, h, wd = x.shape
    g = conv_geom(n, c, h, wd, c, 3, 3, 1, 1)
    rc = lib.nplk_depthwise_bn_act_gap(stream, C.byref(g), _p(x), _p(w), None, _p(mean),
                                       _p(var), _p(gamma), _p(beta), eps, 1, 0.0,
                                       _p(act_out) if act_out is not None else None, _p(gap))
    if rc != 0:
        return rc
    return lib.nplk_softmax(stream, n, c, 1, _p(gap), _p(probs))


def gemm_bias_relu_layer_norm(lib, stream, A, B, Cm, Y, work, ws: int, eps: float = 1e-5,
                              flags: int = 0, between=None) -> int:
    """The large-GEMM workload after its bias fill: Cm = ReLU(A @ B + Cm) with
    Cm holding the per-column bias row in every row on entry (the reference's
    bias through beta = 1 on a pre-filled C, npl_tensor_ops.cpp:115-311, with
    npl_relu applied in the GEMM epilogue), then Y = layer norm of each row of
    Cm (gamma 1, beta 0; npl_activation_norm.cpp:470-522).

    A: [M, K]; B: [K, N]; Cm, Y: [M, N]; work: the GEMM's hi/lo workspace of
    `ws` bytes (nplk_gemm_workspace_size). `between`, if given, is called
    after the GEMM is launched and before the layer norm (a timing event)."""
    M, K = A.shape
    N = B.shape[1]
    rc = lib.nplk_gemm(stream, M, N, K, 1.0, _p(A), K, _p(B), N, 1.0, _p(Cm), N, None, 1, 0.0,
                       flags, _p(work), ws, None)
    if rc != 0:
        return rc
    if between is not None:
        between()
    return lib.nplk_layer_norm(stream, M, N, _p(Cm), _p(Y), None, None, eps)


def fill_bias_rows(Cm, bias) -> None:
    """Cm[i, :] = bias for every row (the pre-fill that carries the bias
    through beta = 1)."""
    Cm.copy_(bias.expand(Cm.shape[0], Cm.shape[1]))
