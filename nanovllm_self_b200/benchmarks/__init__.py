"""Workload generators and benchmark drivers (reference ``scripts/`` and ``pd_self/*/evaluation``)."""
