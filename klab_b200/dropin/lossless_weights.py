"""Top-level name of the reference module `lossless_weights`, served by klab_b200.lossless_weights.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import lossless_weights`
resolves to the B200 implementation."""

from klab_b200.lossless_weights import *  # noqa: F401,F403
from klab_b200 import lossless_weights as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
