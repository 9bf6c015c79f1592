"""B200-native token selection for PagedMoE's decode loop.

Public API:
    make_sampler, make_logits_processors   drop-ins for mlx-lm's factories
    sample_rows, apply_processors, logprobs batched fast paths ([B, V] at once)
    verify                                  draft acceptance of a verify pass
    sampling                                request defaults (pagedmoe/sampling.py)

The CUDA library (libpm_sample.so) is loaded on the first call that launches
work, so host-only modules (settings, request defaults, synthetic workloads)
import without it.  There is no CPU path: that first call raises ImportError
when the library is missing or does not load.
"""

from . import _lib
from . import sampling  # noqa: F401  (host-side defaults, pure Python)
from .params import ProcessorSettings, SamplerSettings  # noqa: F401
from .engine import apply_processors, argmax_confidence, logprobs, sample_rows  # noqa: E402,F401
from .sample_utils import make_logits_processors, make_sampler  # noqa: E402,F401
from .verify import verify  # noqa: E402,F401

__version__ = "0.2.0"


def load_library():
    """Load libpm_sample.so now (building it first when nvcc is present)."""
    return _lib.load()


def library_path() -> str:
    return _lib._build.SO
