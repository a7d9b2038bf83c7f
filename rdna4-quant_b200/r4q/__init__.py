"""r4q — B200 (sm_100a) decode hot path of rdna4-quant.

The compute lives in ``libr4q.so`` (CUDA C++, C ABI declared in
``include/r4q.h``); this package only binds it.  There is no CPU fallback:
importing ``r4q.lib`` raises if the library is missing.
"""
