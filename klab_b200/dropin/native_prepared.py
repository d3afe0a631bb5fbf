"""Top-level name of the reference module `native_prepared`, served by klab_b200.native_prepared.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import native_prepared`
resolves to the B200 implementation."""

from klab_b200.native_prepared import *  # noqa: F401,F403
from klab_b200 import native_prepared as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
