"""Speculative decoding (forgeserve/speculative.py) is not on the pipeline-parallel path this package rebuilds.

The names stay importable so that code importing them from the package keeps loading; calling them raises."""


def verify_draft(*args, **kwargs):
    raise NotImplementedError("speculative decoding is not part of forgeserve_b200 (pipeline-parallel path only)")


def speculative_generate(*args, **kwargs):
    raise NotImplementedError("speculative decoding is not part of forgeserve_b200 (pipeline-parallel path only)")
