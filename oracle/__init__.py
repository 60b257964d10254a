"""TEST INFRASTRUCTURE ONLY: CPU oracle for RF-DETR's Hungarian matching step.

* ``oracle.cost``     numpy float32 restatement of the reference cost chain
                      (kernels_matcher.py:237-264);
* ``oracle.lsap``     ctypes binding of ``lsap.c``, a C restatement of SciPy's
                      ``rectangular_lsap`` (called by the reference at
                      kernels_lap.py:370-379 and patches.py:213-229);
* ``oracle.matcher``  the whole ``HungarianMatcher.forward`` step on the CPU;
* ``oracle.cpu_path`` the reference's CPU path as it runs in training (torch CPU
                      op chain plus SciPy on a thread pool), used only as the
                      timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke`` and ``bench.py``'s CPU-baseline and
reference legs import this package; the product library never does.
"""
