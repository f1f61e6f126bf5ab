"""CPU: argument handling of eigsh on matrix-free operators (no GPU call).

An operator reaches the solver only through y = A x, so the options that need
the matrix itself are refused before any device work: shift-invert (its inner
CG multiplies by A), the fp32 copy of the values, the row renumbering.
"""
import numpy as np
import pytest
import scipy.sparse as sp


def _op(n=50):
    from scipy.sparse.linalg import aslinearoperator

    return aslinearoperator(sp.diags(np.arange(1.0, n + 1)).tocsr())


def test_operator_classification():
    from gpu_eigsh import CudaOperator, operators

    assert operators.is_operator(_op())
    assert not operators.is_operator(sp.eye(4, format="csr"))
    assert not operators.is_operator(np.eye(4))
    assert operators.is_operator(CudaOperator(4, lambda x: x, device="cuda:0"))


@pytest.mark.parametrize("kw, exc", [({"sigma": 0.0}, NotImplementedError), ({"mixed": True}, ValueError),
                                     ({"reorder": True}, ValueError)])
def test_operator_refuses_matrix_options(kw, exc):
    import gpu_eigsh

    with pytest.raises(exc):
        gpu_eigsh.gpu_eigsh(_op(), k=3, **kw)


def test_operator_plan_refuses_comm_and_mixed():
    import gpu_eigsh

    with pytest.raises(ValueError):
        gpu_eigsh.EigshPlan(_op(), mixed=True)
