"""Top-level name of the reference module `autotune` (research/l2-prefetch/src/autotune.py),
served by klab_b200.prefetch_autotune.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import autotune`
resolves to the B200 implementation."""

from klab_b200.prefetch_autotune import *  # noqa: F401,F403
from klab_b200 import prefetch_autotune as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
