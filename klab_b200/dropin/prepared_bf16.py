"""Top-level name of the reference module `prepared_bf16`, served by klab_b200.prepared_bf16.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import prepared_bf16`
resolves to the B200 implementation."""

from klab_b200.prepared_bf16 import *  # noqa: F401,F403
from klab_b200 import prepared_bf16 as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
