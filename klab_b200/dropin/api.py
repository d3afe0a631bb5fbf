"""Top-level name of the reference module `api` (research/l2-prefetch/src/api.py),
served by klab_b200.prefetch_api.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import api`
resolves to the B200 implementation."""

from klab_b200.prefetch_api import *  # noqa: F401,F403
from klab_b200 import prefetch_api as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
