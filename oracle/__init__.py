"""CPU oracle for the fused-expert hot path. TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may use it, and only as the checker / the timed CPU
baseline, never as the thing measured or shipped.

Contents
--------
* ``nf4``  -- the NF4 codec (codebook, blockwise quantize, 2-nibble packing,
  dequantize), restated from the QLoRA paper (Dettmers et al. 2023,
  arXiv:2305.14314, Appendix E) and from the reference's call sites
  (``experts4bit_qlora/_vendor/experts.py:398-457``). bitsandbytes itself is not
  in this container; its published algorithm is restated, not its code.
* ``moe``  -- the reference's per-expert loop (``_vendor/experts.py:468-516``),
  its LoRA wrapper (``lora.py:251-256, 329-460``), the fused driver's
  permutation and combine (``engines/fast.py:125-135, 260-278``), the router
  rule (``engines/cpu_router.py:100-119``) and the FP8 128x128 block dequant
  (``formats/fp8_blocks.py:60-128``), restated in torch/numpy on CPU.
* ``bnb_shim`` -- a stand-in ``bitsandbytes`` package whose codec is ``nf4``
  above, so the reference's own Python can be imported in the build container
  to produce the golden fixtures under ``tests/golden/``.

Parity pinning: the reference's hot-path Python (loop, LoRA, router, combine,
permutation) is pinned by golden vectors produced by running the reference
itself (``tests/golden/make_golden.py``). The NF4 codebook is pinned against
the paper's published table AND its quantile construction. Byte-level parity
with bitsandbytes' quantizer (tie rule at exact midpoints) is unpinned: no
bitsandbytes build exists here, and the reference ships no NF4 byte vectors.
Both the kernel and the oracle consume the same packed bytes, so this affects
input generation only.
"""
