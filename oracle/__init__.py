"""CPU oracles of the reference's hot-path arithmetic.

TEST INFRASTRUCTURE ONLY.  Modules here restate the reference's algorithms
(each function cites the reference file:line it follows) so the sm_100a
kernels can be checked against them.  Only tests/, __graft_entry__.smoke()
and bench.py's cpu-baseline / reference arm may import this package; the
product package (vllm-qdq-plugin_b200/vllm_qdq_plugin) never does.
"""
