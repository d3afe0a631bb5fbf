"""Top-level name of the reference module `packed_fp32`, served by klab_b200.packed_fp32.

Put klab_b200/dropin on sys.path ahead of the reference tree and `import packed_fp32`
resolves to the B200 implementation."""

from klab_b200.packed_fp32 import *  # noqa: F401,F403
from klab_b200 import packed_fp32 as _impl

globals().update({k: v for k, v in vars(_impl).items() if not k.startswith("__")})
