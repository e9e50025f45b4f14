"""CPU oracle: a numpy restatement of the reference's denoiser math (jhanssen/mako-image).

TEST INFRASTRUCTURE ONLY. Nothing in the product (the CUDA library, its C ABI, the C++ host shim) imports, links or
calls anything here; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs use it,
and only as the checker or the timed CPU baseline.

Pinning: the sampler restatement (er_sde.py) is pinned to the reference's own golden vectors
(tests/er_sde_test.cpp:46-56) and to the reference's er_sde.cpp compiled here (oracle/_ref). The transformer math
(qwen_dit.py, ops.py) is "parity unpinned": the reference's golden tensors for it are not shipped
(README.md:261-262) and its GPU kernels (mako-common) are absent, so it is restated from the call sites cited in
each function.
"""
