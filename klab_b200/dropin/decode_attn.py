"""Top-level name of the reference module `decode_attn` (research/l2-prefetch/src),
served by klab_b200.decode_attn."""

from klab_b200.decode_attn import *  # noqa: F401,F403
from klab_b200 import decode_attn as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
