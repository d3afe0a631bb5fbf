"""Top-level name of the reference module `prepared_kernels`, served by klab_b200.prepared_kernels.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import prepared_kernels`
resolves to the B200 implementation."""

from klab_b200.prepared_kernels import *  # noqa: F401,F403
from klab_b200 import prepared_kernels as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
