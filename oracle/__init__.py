"""CPU oracle of the causal-fast block forward -- TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU) restatement of the reference block path of yahavb/lingbot-world-v2,
following the reference's rounding points. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference leg may import it, and only as the checker or the timed CPU
baseline. The product path (the lingbot-world-v2_b200 package) never imports it and has no CPU
fallback.

Pinning: tests/test_oracle_golden.py checks this restatement against fixtures produced by the
reference's own CausalWanAttentionBlock.forward run on CPU (tests/golden/make_golden.py).
The MXFP8 emulation (oracle.mx) is written from the OCP Microscaling Formats v1.0 spec because the
reference's MX arithmetic lives in the un-vendored Neuron library nkilib
(kernels/ffn_mx.py:14-15); MX parity is therefore pinned only to that spec.
"""
