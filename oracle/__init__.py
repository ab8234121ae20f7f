"""CPU oracle for the NVFP4/FP8 paged-attention path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only
as the checker or the timed CPU baseline.  The product path
(``qwarz_b200``) never imports it and has no CPU fallback.

Modules
  nvfp4      E2M1/E4M3 rounding, the NVFP4 page writer, the dequant gather
             (restates src/qwasar_runtime/xqa.py:73-143), the FP8 shadow cast
             (engine/forward/draft.py:209-210)
  attention  FP32 softmax attention with the reference's lower-right causal
             mask and GQA (restates xqa.py:612-673), the draft split-K and
             its LSE merge (engine/forward/draft_attention.py:23-79)
  k8v4       the K8/V4 quantised cache (bit planes, Hadamard-rotated
             blocks, the reader formula of the reference's K8/V4 design) and
             FP32 attention over it
  rng        a version-independent seeded byte/float stream for fixtures

Pinning.  The dequant and the attention are pinned by golden vectors that
tests/golden/make_golden.py produced from the reference's own kernels
(Triton interpreter on CPU) and its SDPA oracle path; the FP8 shadow cast is
pinned by a table of the reference expression over every FP16 value.  The
NVFP4 *writer* is a third-party kernel absent from the reference tree
(ExLlamaV3 ``_paged_kv_update_nvfp4_kernel`` @ 63b32f0); its bytes are
"parity unpinned" and the writer here restates the rule written in
nvfp4.py (amax/6 scale, RNE E4M3 and E2M1).
"""
