"""Top-level name of the reference module `dynamic_projection`, served by klab_b200.dynamic_projection.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import dynamic_projection`
resolves to the B200 implementation."""

from klab_b200.dynamic_projection import *  # noqa: F401,F403
from klab_b200 import dynamic_projection as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
