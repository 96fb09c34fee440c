"""CPU oracle for the operator-dispatch hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package.  It is the checker, never the thing
measured or shipped: the product (``spirv_inference_b200``) never imports it.
"""
