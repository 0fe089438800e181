"""Eviction policies selectable by name through ``pool._policy_factory``.

Each module mirrors a policy of bigrig_engine/policies/ with the same decisions
on the same request stream (miss counts are pinned by tests/golden/), written
against the contract in ``bigrig_b200.pool.Policy``.
"""
