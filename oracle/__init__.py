"""CPU oracle of the Qwen3.6-MoE expert block -- TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s
CPU-baseline leg. The shipped library (``flowmoe``) never imports this package.
"""
