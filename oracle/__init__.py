"""CPU oracle for the byteprof decode hot path -- TEST INFRASTRUCTURE ONLY.

A plain numpy restatement of the reference's algorithms for the skinny linear (bf16 and int8
weight-only) and the fused mLSTM recurrence. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it, and only as the checker or the
timed CPU baseline: the product package `byteprof_b200` never imports it.

Pinning: `tests/golden/make_golden.py` runs the reference's own code in the development container
(its torch quantizer and dequantizer, and its Triton kernels under the Triton CPU interpreter where
the interpreter supports them) and stores the results under `tests/golden/`; `tests/test_oracle_golden.py`
checks this oracle against them. The bf16 variants of the mLSTM recurrence cannot run in the
Triton interpreter (it has no bf16); there the oracle follows the reference's casts as stated in
`oracle/mlstm_ref.py`, derived from Triton 3.6's type-promotion rules.
"""
