"""Shared helpers: golden fixtures and the parity metrics.

Parity metrics (one EM iteration unless stated), all computed against the fp64
restatement of the reference algorithm (``oracle.flash_em_fused_f64``):

* ``mu``: max |Δmu| / max(|mu|, sqrt(var))   -- scale-aware relative error: the
  plain relative error is meaningless for means that happen to sit near zero.
* ``var``: max |Δvar| / var
* ``log_pi``: max |Δlog_pi| (= relative error of pi)
* ``ln``: max |Δlog_normalizer| (absolute)

Components whose responsibility mass n_k / N is below ``mass_floor`` are
excluded from the mu/var metrics (their mean and variance are set by a handful
of points with weights ~1e-30 and are ill-conditioned in any fp32 evaluation).
"""
import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_names(prefix=""):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def param_errors(got, ref64, n_k=None, N=None, mass_floor=1e-4):
    """got/ref64: (mu, var, log_pi, ln) arrays.  Returns dict of max errors."""
    mu, var, lp, ln = [np.asarray(a, np.float64) for a in got]
    rmu, rvar, rlp, rln = [np.asarray(a, np.float64) for a in ref64]
    keep = np.ones(rmu.shape[0], bool)
    if n_k is not None and N is not None:
        keep = (np.asarray(n_k) / N) > mass_floor
    scale = np.maximum(np.abs(rmu), np.sqrt(rvar))
    e = {
        "mu": float(np.max((np.abs(mu - rmu) / scale)[keep], initial=0.0)),
        "var": float(np.max((np.abs(var - rvar) / rvar)[keep], initial=0.0)),
        "log_pi": float(np.max(np.abs(lp - rlp)[keep], initial=0.0)),
        "ln": float(np.max(np.abs(ln - rln), initial=0.0)),
    }
    return e
