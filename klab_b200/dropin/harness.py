"""Top-level name of the reference module `harness` (research/l2-prefetch/src/harness.py),
served by klab_b200.prefetch_harness.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import harness`
resolves to the B200 implementation."""

from klab_b200.prefetch_harness import *  # noqa: F401,F403
from klab_b200 import prefetch_harness as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
