"""CPU oracle for the TinyLlama INT8 hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports, links or
executes anything under ``oracle/``; only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and
only as the checker (or as the timed CPU baseline), never as the thing
measured or shipped.

Modules
-------
golden       NumPy restatement of the reference INT8 bridge golden model
             (model/tinyllama_gemm_int8.py, model/tinyllama.py).
weights      Seed-generated random TinyLlama archives in the reference's
             ``TinyLlamaWeights`` npz key schema, plus INT8 weight quantization.
kv_golden    KV-cached restatement built from the golden's own blocks: the
             semantics the B200 engine implements (INT8 KV cache, per-row
             activation scales during decode).
contract     Fixed-point contracts pinned by the RTL and the trace exporter:
             Q16.16 requantize, Q16.16 RoPE rounding, argmax tie rule, stop
             priority, KV-cache addressing.

Parity status: pinned. ``tests/golden/make_fixtures.py`` runs the reference's
own Python modules (in the build container, where the reference is mounted)
and stores their outputs as fixtures; ``tests/test_oracle_*.py`` check this
restatement against those fixtures and against the committed ``sim/`` KATs.
"""
