"""Top-level name of the reference module `cuda_module`, served by klab_b200.cuda_module.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import cuda_module`
resolves to the B200 implementation."""

from klab_b200.cuda_module import *  # noqa: F401,F403
from klab_b200 import cuda_module as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
