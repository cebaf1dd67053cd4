"""CPU oracle for the paged-KV speculative-decoding path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithm (sup-zzj/speculative-decoding-lab,
files cited per function).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline; the product (``engine``,
``specdec``, ``libsdl_b200.so``) never routes through it.

Parity pin: every module is checked against golden fixtures produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference and
records its outputs) in ``tests/test_oracle_golden.py``.

Modules:
  kv         -- BlockAllocator / PagedKVCache (engine/kv.py:45-205)
  attention  -- gather + softmax attention (engine/attention.py:41-215)
  sampler    -- logits_to_probs, acceptance, residual, the defined integer
                inverse-CDF draw, batch_accept (specdec/sampler.py:19-92,
                engine/spec_scheduler.py:41-88)
  model      -- numpy Qwen2/toy decoder forward over the oracle cache
                (engine/model.py, engine/qwen.py)
  scheduler  -- continuous and speculative schedulers (engine/scheduler.py,
                engine/spec_scheduler.py)
"""
