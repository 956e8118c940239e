"""B200-native (sm_100a) streaming Taylor-moment + block-coreset causal attention.

Drop-in for the fast path of PositiveLoss/streaming-attention
(``fast_article_attention.py``): the same entry points and arguments, computed
by hand-written CUDA kernels in ``libsa_b200.so`` through a C ABI
(``include/streaming_attention.h``), plus the streaming (decode) class
``ArticleStreamingAttention`` of ``streaming_taylor_coreset_attention.py``
and the segment-mean variant of ``triton_article_attention.py``
(``triton_article_causal_attention``).  There is no CPU compute path.
"""

from .fast import (  # noqa: F401
    BlockReps,
    FastArticleStats,
    build_completed_block_reps,
    classical_causal_attention,
    exp_taylor,
    fast_article_causal_attention,
    fast_article_causal_attention_single,
    num_taylor_features,
    safe_relative_l2,
)

from .streaming import ArticleStreamingAttention, AttentionQueryStats  # noqa: F401
from .segment import (  # noqa: F401
    TritonArticleStats,
    build_segment_mean_coreset,
    torch_classical_causal_attention,
    triton_article_causal_attention,
    triton_flash_causal_attention,
)

__version__ = "0.1.0"
