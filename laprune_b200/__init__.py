"""laprune_b200 -- B200-native (sm_100a) implementation of LAPrune's
sparse-decode hot path, behind the reference's own Python surface.

* ``laprune_b200.ops``        fused decode step (LUT build -> scorer -> exact
                               top-k -> GQA gather + split-K flash-decode)
* ``laprune_b200.synthetic``  seeded inputs in the benchmark shapes
* ``laprune_b200.build``      in-tree nvcc build of the C-ABI library

The CUDA library is loaded lazily on first use; nothing here falls back to
a CPU implementation.
"""
__version__ = "0.1.0"
