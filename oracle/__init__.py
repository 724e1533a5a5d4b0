"""CPU oracle for the sonic-moe FP8 MoE-layer forward path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``sonic-moe_b200/``) imports this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may use it, and only as the checker or as the timed CPU
restatement of the reference -- never as the thing measured for the GPU arm.

Modules and what pins them:

* ``mathfn``   -- float32 ``exp`` / ``log`` with a fixed operation order (Cody-Waite reduction +
  Taylor polynomial; frexp + atanh series).  The CUDA router uses the same sequence of IEEE
  single operations, so routing scores are bit-exact between the two.
* ``routing``  -- restatement of the reference top-k router
  (``sonicmoe/functional/topk.py:143-260``): index bits written into the low mantissa bits,
  descending order with ties to the lower expert, softmax over the top-k, or log-softmax ->
  top-k -> exp (+renorm).  PINNED: against the reference's own torch routing
  (``sonicmoe/functional/forward.py:128-141``) on the committed golden vectors
  (``tests/golden/``), plus known-answer tie cases derived from ``topk.py:200-234``.
* ``metadata`` -- restatement of ``tests/metadata_test.py:17-70`` (stable argsort by expert),
  plus this build's 128-row padded expert layout.  PINNED: against outputs of the reference's own
  pure-torch metadata functions, committed as golden vectors.
* ``quant``    -- the e4m3 quantiser this build defines (1x128 activation groups, 128x128 weight
  blocks, power-of-two UE8M0 scales).  The reference has NO FP8 quantiser
  (grep for fp8/e4m3/quant in ``sonicmoe/`` finds nothing numeric), so this part is
  "parity unpinned": it is a specification, checked only against torch's float8 conversion.
* ``layer``    -- the reference's eager MoE math (``sonicmoe/moe.py:278-360`` and the per-expert
  loop of ``benchmarks/moe-cute.py:204-244`` for top-k-over-softmax and the concat layout), in a
  dense variant and a fake-quantised FP8 variant.  The dense variant is PINNED against the
  reference ``MoE.forward(kernel_backend_moe=torch)`` outputs in ``tests/golden/``.
"""
