"""kvdlra_b200 -- kvdlra's streaming compressed-KV path on B200 (sm_100a).

Public surface (drop-in for kvdlra's):
* :class:`BugStreamingCache`, :class:`BugStreamingLayer` -- the HuggingFace
  cache (src/kvdlra/cache/bug_cache.py);
* :func:`augmented_bug_step`, :func:`blocked_bug_subspace`,
  :func:`blocked_bug_project` -- the integrator (streaming_torch.py);
* :class:`BUGPress` -- the prefill low-rank press (src/kvdlra/press/bug_press.py);
* :mod:`kvdlra_b200.accounting` -- the float-equivalent charge (accounting.py);
* :func:`enable_factored_decode` -- a model's decode attention answered by the
  factored kernel over the compressed cache;
* :mod:`kvdlra_b200.harness` -- chunked prefill and greedy decode drivers.

The compute runs in ``_lib/libkvdlra_b200.so`` (built by
``python -m kvdlra_b200.build``); it is loaded on first use.
"""

from .cache import BugStreamingCache, BugStreamingLayer, RopeAngles
from .integrator import augmented_bug_step, blocked_bug_project, blocked_bug_subspace
from .press import BUGPress
from .attention import enable_factored_decode

__all__ = [
    "BugStreamingCache", "BugStreamingLayer", "RopeAngles",
    "augmented_bug_step", "blocked_bug_project", "blocked_bug_subspace", "BUGPress",
    "enable_factored_decode",
]
__version__ = "0.1.0"
