"""CPU oracle for the ExecutionPlan runtime -- TEST INFRASTRUCTURE ONLY.

A plain-NumPy restatement of the reference's runtime path, used as the
checker for the B200 backend.  Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may
import it; the product (the ``backend.hal_cuda`` HAL and its kernels) never
does, and fails loudly instead of falling back to it.

Modules and what each restates:

* ``hal_numpy``  -- NumpyBackend (backend/hal_numpy.py:12-189) on top of the
  vendor-SDK byte model (backend/dpu_sdk.py:44-191);
* ``lowering``   -- the host-star redistribute primitives
  (comm/lowering.py:38-194): sequential in-dtype sums in rank order,
  merges by global range;
* ``kernels``    -- NumPy kernel stubs for every op of the step graph, with
  the bf16 rounding points of HF ``LlamaForCausalLM``.

Parity is pinned by golden vectors generated from the reference itself
(tests/golden/make_golden.py): the comm-plan segment tables, the redistribute
outputs (bit-exact, bf16 and fp32), the KV layout tables and HF logits /
greedy tokens for the tiny configuration.
"""
