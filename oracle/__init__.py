"""CPU oracle for the paged decode / speculative-verify hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) may import it, and
they use it as the checker / the timed CPU reference, never as the product
path.

Contents (numpy restatements of the reference, henry-tmp-de/specdec-nanovllm):

* ``attention``  -- paged decode attention (``nanovllm/kernels/paged_decode_attn.py:472-495``)
  extended to k+1 causal verify rows with flash-attn's bottom-right alignment
  (``nanovllm/layers/attention.py:64-70`` with the metadata of
  ``nanovllm/engine/model_runner.py:522-548``).
* ``quant``      -- ``quantize_weight`` / ``dequantize_weight`` / the W8A16 reference
  product (``nanovllm/layers/quant.py:123-159``).
* ``verify``     -- ``verify_batch`` rejection sampling with injected uniforms and
  exponentials (``nanovllm/spec_decode/verify.py:42-209``).
* ``philox``     -- Philox4x32-10 (Salmon et al., SC'11) and the fixed-operation
  float32 logarithm that the GPU sampler mirrors bit for bit.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
fixtures produced by running the reference's own Python code
(``tests/golden/make_golden.py``) and against the reference's known-answer
tests (``tests/test_spec_decode.py`` cases 2A/2B/2C/3/5/6 and
``tests/test_temp_broadcast.py`` of the reference).
"""
