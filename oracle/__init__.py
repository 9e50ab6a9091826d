"""CPU oracle for the paged-KV attention path -- TEST INFRASTRUCTURE ONLY.

A restatement, on the CPU, of the reference engine's own path
(shubhav1/my-inference-engine): the Python KVCache with its tail-popped free
list, slot mapping and dense gather (kv_cache.py:8-121), RoPE with bf16
rounding after every op (model.py:58-65, :148-155), and attention as fp32
SDPA over the gathered K/V with a bottom-right causal mask (model.py:104-107,
:186-195; kernels/test_fa2.py:28-35).

Pinned against the reference itself: tests/golden/make_golden.py runs the
reference checkout on the CPU and stores its outputs (block tables, free
lists, slot mappings, bf16 bit patterns of roped q/k and written pool slots,
fp32 attention outputs of the reference's kernel-test cases and BASELINE
configs 0/1, greedy ids of the full model); tests/test_oracle_golden.py checks
this package against every fixture.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import it, and only as the checker or the timed CPU baseline --
never on the product path.
"""
