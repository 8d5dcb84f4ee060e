"""tabby_b200: B200-native (sm_100a) token sampler, a drop-in for the GPU sampling path
of xOAviOx/tabby (src/engine/sampler.ts + the reduce_max / reduce_sumexp / topk_partial /
topk_select kernels driven by src/engine/forward.ts:520-601)."""
from .sampler import (  # noqa: F401
    DEFAULT_SAMPLING,
    MAX_TOP_K,
    SampleBatch,
    SampleOutcome,
    Sampler,
    SamplingParams,
    SeededRandom,
    TopKResult,
    decode_sample_block,
    pool_size,
    sampleFromTopK,
    sample_from_topk,
)
