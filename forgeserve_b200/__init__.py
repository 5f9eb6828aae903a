"""forgeserve_b200: the pipeline-parallel forward path of forgeserve, rebuilt for B200 (sm_100a)."""
