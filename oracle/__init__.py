"""CPU oracle of the reference's per-denoising-step attention path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs may import this package, and only as the
checker (or as the timed CPU restatement of the reference). The product
(dllm-serve_b200/dllmserve_b200) never imports it and has no CPU fallback.

Parity pin: the restatement is checked against golden vectors produced by
running the reference's own ``dllmserve.layers.attention`` module on CPU
(tests/golden/make_golden.py, fixtures in tests/golden/*.npz).
"""
