"""Shared helpers: golden fixtures and the parity metrics.

Parity metrics (one EM iteration unless stated), all computed against the fp64
restatement of the reference algorithm (``oracle.flash_em_fused_f64``):

* ``mu``: max |Δmu| / max(|mu|, sqrt(var))   -- scale-aware relative error: the
  plain relative error is meaningless for means that happen to sit near zero.
* ``var``: max |Δvar| / var over well-conditioned components (n_k >= 2 and
  var >= 1e-3 (mu^2 + var)); plus ``var_abs`` = max |Δvar| / (mu^2 + var) over
  all of them -- var is evaluated as sq/n - mu^2, a difference of two numbers of
  size mu^2 + var, so for degenerate components (one point, var at the 1e-6
  floor) any fp32 evaluation, the reference's included, only fixes it to
  ~1e-7 (mu^2 + var).
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


def em_golden_names():
    """The one-iteration flash_em_fused fixtures (config slices and ragged edge cases)."""
    return [n for n in golden_names() if n.startswith(("c1_iter", "c2_slice", "c3_slice", "c4_slice",
                                                         "c5_slice", "edge_"))]


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def param_errors(got, ref64, n_k=None, N=None, mass_floor=1e-4):
    """got/ref64: (mu, var, log_pi, ln) arrays.  Returns dict of max errors."""
    mu, var, lp, ln = [np.asarray(a, np.float64) for a in got]
    rmu, rvar, rlp, rln = [np.asarray(a, np.float64) for a in ref64]
    keep = np.ones(rmu.shape[0], bool)
    cond = np.ones(rmu.shape, bool)
    if n_k is not None and N is not None:
        nk = np.asarray(n_k)
        keep = (nk / N) > mass_floor
        cond = (keep & (nk >= 2.0))[:, None] & (rvar >= 1e-3 * (rmu ** 2 + rvar))
    scale = np.maximum(np.abs(rmu), np.sqrt(rvar))
    e = {
        "mu": float(np.max((np.abs(mu - rmu) / scale)[keep], initial=0.0)),
        "var": float(np.max((np.abs(var - rvar) / rvar)[cond], initial=0.0)),
        "var_abs": float(np.max((np.abs(var - rvar) / (rmu ** 2 + rvar))[keep], initial=0.0)),
        "log_pi": float(np.max(np.abs(lp - rlp)[keep], initial=0.0)),
        "ln": float(np.max(np.abs(ln - rln), initial=0.0)),
    }
    return e
