"""Prints the directory of an OpenBLAS shared object (libopenblas*.so) found
among this Python's site-packages, for oracle/Makefile's BLAS_DIR default.
Test infrastructure: the reference's `make blas` build needs cblas_sgemm and
this image has no system OpenBLAS. Prints nothing when none is found."""
import glob
import os
import site
import sys

roots = list(dict.fromkeys(site.getsitepackages() + [site.getusersitepackages()] + sys.path))
for root in roots:
    if not root or not os.path.isdir(root):
        continue
    hits = sorted(glob.glob(os.path.join(root, "*", "libopenblas*.so")))
    if hits:
        print(os.path.dirname(hits[0]))
        break
