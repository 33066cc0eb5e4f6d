"""B200 (sm_100a) kernels for the Granite Speech NAR Conformer conv module, behind the reference's
``torch.library`` op names (``granite::dwconv_silu``, ``granite::dwconv_silu_glu``) plus whole-module ops, and the
rest of the Conformer block (feed-forward halves, block-local attention, post norm).

Importing the package registers the ops; the CUDA library itself is loaded on the first call and its absence is
an error, never a fallback.
"""
from . import ops  # noqa: F401  registers the granite:: custom ops
from .conv_kernel import enable_dwconv_silu  # noqa: F401
from .dispatch import Chunk, bucket_frames, plan_chunks, shard_chunks  # noqa: F401
from .block import (ConformerEncoderStack, PreparedConformerBlock, prepare_block_from_params,  # noqa: F401
                    prepare_conformer_block, run_conformer_block)
from .encoder import GraniteCTCEncoder  # noqa: F401
from .stack import ConvModuleStack  # noqa: F401
from .weights import (PreparedConvModule, fold_conv_bn_, glu_interleave, prepare_conv_module,  # noqa: F401
                      prepare_from_params, prepare_from_tensors, quantize_per_channel)

__version__ = "1.0.0"
