"""bigrig_b200: BigRig's MoE expert hot path on NVIDIA B200 (sm_100a).

Drop-in Python surface of the reference engine's expert path:

* ``pool``      -- eviction-policy contract, baselines, resolver, replay tools
                   (bigrig_engine/pool.py); ``policies/`` -- LFUDA (default), ARC,
                   LIRS, S3-FIFO, GateRank, CoAct (bigrig_engine/policies/).
* ``stream``    -- ExpertPool on an HBM slab, StreamingSwitchGLU, attach,
                   StreamHandle (bigrig_engine/stream.py).
* ``fetch``     -- pinned host expert store with the fetcher interface
                   (bigrig_engine/fetch.py).
* ``layered``   -- the layer-major prefill schedule (bigrig_engine/layered.py).
* ``block``     -- the MoE block around the layer: router, call, combine.
* ``ops``       -- torch wrappers of the C ABI in include/bigrig_b200.h, served by
                   the sm_100a kernels of libbigrig_b200.so.  No CPU fallback.
"""
__version__ = "0.1.0"
