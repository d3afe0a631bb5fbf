"""Top-level name of the reference example `kv_pair_projection` (examples/), served
by klab_b200.kv_pair: prepare_pair_graph with the same contract."""

from klab_b200.kv_pair import prepare_pair_graph  # noqa: F401
