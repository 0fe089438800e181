"""Eviction policies selectable by name through ``pool._policy_factory``.

Built here: LFUDA (the default), GateRank, S3-FIFO and ARC, each making the
decisions of its namesake in bigrig_engine/policies/ on the same request stream
(miss counts are pinned by tests/golden/), with per-expert state held as columns
(``_columns``).  Any other module that follows ``bigrig_b200.pool.Policy`` plugs in
by its dotted module path.
"""
