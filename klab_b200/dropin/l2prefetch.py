"""Top-level name of the reference module `l2prefetch`, served by klab_b200.l2prefetch.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import l2prefetch`
resolves to the B200 implementation."""

from klab_b200.l2prefetch import *  # noqa: F401,F403
from klab_b200 import l2prefetch as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
