"""ORACLE -- test infrastructure, not product code.

CPU restatements of the reference's reverse-flow denoising path, each function
citing the reference file:line it follows. Only tests/, __graft_entry__.smoke()
and the CPU-baseline leg of bench.py may import this package, and only as the
checker. The product (the flow2surf_b200 package and its CUDA library) never
imports or calls anything here.

    native     -- bit-exact C restatements (KNN, nearest distance, FPS)
    model      -- NumPy restatement of Flow2SurfNet (float64 by default)
    inference  -- NumPy/SciPy restatement of patch_denoise and Chamfer
"""
