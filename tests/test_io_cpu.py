"""Matrix Market reader / writer (host code of the library, no GPU) against
scipy.io's reader and writer."""
import numpy as np
import pytest
import scipy.io
import scipy.sparse as sp

from gpu_eigsh.io import mmread, mmwrite


def _rand_sym(n, seed):
    rng = np.random.default_rng(seed)
    A = sp.random(n, n, density=0.05, random_state=np.random.RandomState(seed), format="csr")
    A = A + A.T + sp.diags(rng.standard_normal(n))
    return A.tocsr()


def test_roundtrip_exact_and_scipy_compatible(tmp_path):
    A = _rand_sym(300, 0)
    A.data *= np.pi * 1e-7            # values that "%.15e" would not round-trip
    f = tmp_path / "a.mtx"
    mmwrite(f, A)
    B = mmread(f)
    assert (abs(A - B) > 0).nnz == 0 and np.array_equal(A.indptr, B.indptr)
    C = scipy.io.mmread(str(f)).tocsr()
    assert (abs(A - C) > 0).nnz == 0
    g = tmp_path / "s.mtx"
    mmwrite(g, A, symmetric=True)
    assert (abs(mmread(g) - A) > 0).nnz == 0
    assert (abs(scipy.io.mmread(str(g)).tocsr() - A) > 0).nnz == 0


def test_reads_scipy_files_symmetric_pattern_duplicates(tmp_path):
    A = _rand_sym(200, 1)
    f = tmp_path / "sym.mtx"
    scipy.io.mmwrite(str(f), A, symmetry="symmetric")
    assert abs(mmread(f) - A).max() < 1e-12
    p = tmp_path / "pat.mtx"
    p.write_text("%%MatrixMarket matrix coordinate pattern symmetric\n% comment\n3 3 3\n1 1\n2 1\n3 2\n")
    P = mmread(p).toarray()
    np.testing.assert_array_equal(P, [[1, 1, 0], [1, 0, 1], [0, 1, 0]])
    d = tmp_path / "dup.mtx"
    d.write_text("%%MatrixMarket matrix coordinate real general\n2 2 4\n1 2 1.5\n2 1 -2\n1 2 0.25\n2 2 4e0\n")
    D = mmread(d)
    np.testing.assert_array_equal(D.toarray(), [[0, 1.75], [-2, 4]])
    assert D.nnz == 3
    s = tmp_path / "skew.mtx"
    s.write_text("%%MatrixMarket matrix coordinate integer skew-symmetric\n2 2 1\n2 1 3\n")
    np.testing.assert_array_equal(mmread(s).toarray(), [[0, -3], [3, 0]])


def test_errors(tmp_path):
    from gpu_eigsh import LanczosError

    bad = tmp_path / "bad.mtx"
    bad.write_text("%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1.0\n3 1 2.0\n")
    with pytest.raises(LanczosError, match="cannot parse entry 2"):
        mmread(bad)
    short = tmp_path / "short.mtx"
    short.write_text("%%MatrixMarket matrix coordinate real general\n2 2 3\n1 1 1.0\n")
    with pytest.raises(LanczosError, match="fewer entries"):
        mmread(short)
    with pytest.raises(LanczosError, match="cannot read"):
        mmread(tmp_path / "missing.mtx")
    arr = tmp_path / "arr.mtx"
    arr.write_text("%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n")
    with pytest.raises(LanczosError, match="coordinate"):
        mmread(arr)
