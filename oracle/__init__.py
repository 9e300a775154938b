"""CPU oracle for the MoEInfra quantized-expert hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
package. It is used by ``tests/`` (as the checker), by
``__graft_entry__.smoke()`` (as the checker) and by ``bench.py``'s
``cpu_baseline`` leg and ``--impl reference`` arm (as the timed CPU
restatement of the reference's path).

What it restates (all file:line citations are into the reference project
ParshwaPatel-07/MoEInfra):

* ``oracle.nf4``    NF4 unpack / blockwise dequant to bf16 (nested absmax
  included), the two bitsandbytes 0.50.2 linear semantics the reference
  reaches through ``Linear4bit`` (``transfer/nf4_reconstruct.py:9-14``,
  ``:45-54``, ``:94``), the SwiGLU expert (``:152-155``) and a NF4
  quantizer for synthetic stores.
* ``oracle.router`` ``ExpertRouter.route_with_logits``
  (``engine/router.py:65-94``).
* ``oracle.moe``    ``MoELayer._forward_tokens`` dispatch and combine order
  (``model/moe_layer.py:142-191``).

Parity pins: the router and the dispatch/combine are pinned by golden
vectors produced by the reference's own Python code (``tests/golden``).
The NF4 arithmetic lives in bitsandbytes 0.50.2 (``requirements.txt:3``),
which is absent from this environment: its codebook is pinned to the
published QLoRA NF4 table and its dequant to known-answer vectors; the
bitsandbytes kernels themselves could not be run ("parity unpinned" for
bnb's own kernels; see the header of ``oracle.nf4``).
"""
