"""Top-level name of the reference module `half_projection`, served by klab_b200.half_projection.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import half_projection`
resolves to the B200 implementation."""

from klab_b200.half_projection import *  # noqa: F401,F403
from klab_b200 import half_projection as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
