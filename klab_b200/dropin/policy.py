"""Top-level name of the reference module `policy` (research/l2-prefetch/src/policy.py),
served by klab_b200.prefetch_policy.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import policy`
resolves to the B200 implementation."""

from klab_b200.prefetch_policy import *  # noqa: F401,F403
from klab_b200 import prefetch_policy as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
