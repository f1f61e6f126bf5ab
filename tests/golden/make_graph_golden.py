"""Generate golden kNN Laplacians with the reference's own generator script.

    python tests/golden/make_graph_golden.py REFERENCE_ROOT

REFERENCE_ROOT is the root of a checkout of the reference.  Runs
benchmark/generate_large_laplacian.py unmodified (its own argument parser,
cKDTree, scipy assembly and mmwrite) into a temporary directory for a few
small configurations, reads each laplacian.mtx back with scipy.io.mmread and
stores the CSR arrays with the arguments in graph_generator.npz next to this
script (committed; the tests read it without the reference present).

Cases: (n, dim, k, bw, seed) = (250, 10, 15, 0.3, 123)  the script's own
defaults at a small n (the all-pairs search), (400, 2, 10, 0.05, 7) and
(300, 3, 8, 0.1, 11) (the cell-grid search).
"""
from __future__ import annotations

import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import scipy.io
import scipy.sparse as sp

HERE = Path(__file__).resolve().parent
CASES = [(250, 10, 15, 0.3, 123), (400, 2, 10, 0.05, 7), (300, 3, 8, 0.1, 11)]


def main(root: str) -> None:
    script = Path(root) / "benchmark" / "generate_large_laplacian.py"
    out = {}
    for c, (n, dim, k, bw, seed) in enumerate(CASES):
        with tempfile.TemporaryDirectory() as tmp:
            subprocess.run([sys.executable, str(script), "--n", str(n), "--dim", str(dim), "--k", str(k),
                            "--bw", repr(bw), "--seed", str(seed), "--outdir", tmp], check=True,
                           stdout=subprocess.DEVNULL)
            L = sp.csr_matrix(scipy.io.mmread(str(Path(tmp) / "laplacian.mtx")))
        L.sum_duplicates()
        L.sort_indices()
        out[f"c{c}_args"] = np.array([n, dim, k, bw, seed], dtype=np.float64)
        out[f"c{c}_indptr"] = L.indptr.astype(np.int32)
        out[f"c{c}_indices"] = L.indices.astype(np.int32)
        out[f"c{c}_data"] = L.data.astype(np.float64)
    np.savez_compressed(HERE / "graph_generator.npz", ncases=np.array(len(CASES)), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_graph_golden.py REFERENCE_ROOT")
    main(sys.argv[1])
