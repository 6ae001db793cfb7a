"""The reference's six graft GEMMs in its exact operand orientations (numpy, fp32).

TEST INFRASTRUCTURE ONLY (checker for the CUDA library; see oracle/__init__.py).

Each function restates one wrapper of src/graft_ops_impl.inc / src/gemm_impl.inc
in row-major terms.  Operands are optionally rounded to bf16 with the
reference's bias trick first, because the reference converts f32 operands to
bf16 before every rocBLAS call (src/gemm_impl.inc:398-405, 455, 525).
"""
from __future__ import annotations

import numpy as np

from .bitexact import round_bf16


def _op(a, bf16: bool):
    a = np.asarray(a, dtype=np.float32)
    return round_bf16(a) if bf16 else a


def expand_forward(x_h, w_sh, bf16=True):
    """ExpandForward: out[M,S] = x_h[M,H] @ W[S,H]^T (graft_gemm_fwd, gemm_impl.inc:388-445)."""
    return (_op(x_h, bf16).astype(np.float64) @ _op(w_sh, bf16).astype(np.float64).T).astype(np.float32)


def contract_forward(x_i, w_sh, bf16=True):
    """ContractForward: out[M,H] = x_i[M,S] @ W_storage[S,H] (graft_ops_impl.inc:33-114)."""
    return (_op(x_i, bf16).astype(np.float64) @ _op(w_sh, bf16).astype(np.float64)).astype(np.float32)


def expand_weight_grad(x_h, dy_s, bf16=True):
    """ExpandWeightGrad: dW[S,H] = dy[M,S]^T @ x_h[M,H] (grad_gemm, gemm_impl.inc:450-514)."""
    return (_op(dy_s, bf16).astype(np.float64).T @ _op(x_h, bf16).astype(np.float64)).astype(np.float32)


def contract_weight_grad(x_i, dy_h, bf16=True):
    """ContractWeightGrad in storage orientation: dW[S,H] = x_i[M,S]^T @ dy[M,H]
    (grad_gemm_storage_canonical, gemm_impl.inc:520-584)."""
    return (_op(x_i, bf16).astype(np.float64).T @ _op(dy_h, bf16).astype(np.float64)).astype(np.float32)


def expand_input_grad(dy_s, w_sh, bf16=True):
    """ExpandInputGrad: dx_h[M,H] = dy[M,S] @ W[S,H] (layer_backward_impl.inc:311-342)."""
    return (_op(dy_s, bf16).astype(np.float64) @ _op(w_sh, bf16).astype(np.float64)).astype(np.float32)


def contract_input_grad(dy_h, w_sh, bf16=True):
    """ContractInputGrad: gi[M,S] = dy_h[M,H] @ W_storage[S,H]^T (layer_backward_impl.inc:148-155)."""
    return (_op(dy_h, bf16).astype(np.float64) @ _op(w_sh, bf16).astype(np.float64).T).astype(np.float32)
