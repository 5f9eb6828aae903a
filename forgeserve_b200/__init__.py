"""forgeserve_b200: the pipeline-parallel forward path of forgeserve, rebuilt for B200 (sm_100a).

The public names are the reference package's export list (forgeserve/__init__.py:11)."""

from .config import ModelConfig
from .engine import Engine, Request
from .kv import ContiguousKV, new_contiguous_cache
from .model import ForgeModel
from .paged import BlockAllocator, OutOfBlocks, PagedKVPool
from .parallel import SINGLE, TPContext
from .pipeline import PipelineStage, PipelineState, bubble_fraction, pipeline_forward, pipeline_generate, stage_layers
from .pipeline_engine import PipelineEngine
from .sampling import generate, sample
from .speculative import speculative_generate, verify_draft

__all__ = ["PipelineStage", "PipelineState", "bubble_fraction", "pipeline_forward", "pipeline_generate", "stage_layers",
           "speculative_generate", "verify_draft", "Engine", "Request", "BlockAllocator", "OutOfBlocks", "PagedKVPool",
           "ModelConfig", "ForgeModel", "TPContext", "SINGLE", "ContiguousKV", "new_contiguous_cache", "generate",
           "sample"]
