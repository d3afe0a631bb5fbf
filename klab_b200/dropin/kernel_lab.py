"""Top-level name of the reference module `kernel_lab`, served by klab_b200.kernel_lab.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import kernel_lab`
resolves to the B200 implementation."""

from klab_b200.kernel_lab import *  # noqa: F401,F403
from klab_b200 import kernel_lab as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
