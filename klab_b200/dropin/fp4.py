"""Top-level name of the reference module `fp4`, served by klab_b200.fp4.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import fp4`
resolves to the B200 implementation."""

from klab_b200.fp4 import *  # noqa: F401,F403
from klab_b200 import fp4 as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
