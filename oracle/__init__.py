"""CPU oracle for the B200 rasterizer — TEST INFRASTRUCTURE, not the product.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline /
``--impl reference`` legs import this package, and only as the checker or the
timed CPU baseline. The product path (torch_gsplat_bridge_fast) never imports it.

Parity pinning: the torch restatements in ``torch_ref`` and the C restatement in
``gsplat_oracle.c`` are checked against golden vectors produced by running the
reference's own torch functions (``tests/golden/make_golden.py``, run where the
reference checkout is mounted). The reference's binning exists only as Metal
kernels; its restatement is pinned by the property that compositing through
the binned lists reproduces the reference's dense torch renderer exactly.
"""
