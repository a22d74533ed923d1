"""CPU oracle for the packed LayerSkip-Llama draft/verify step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``thesis_b200``) imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and the CPU
baseline legs of ``bench.py`` use it.  It restates, in numpy, the arithmetic of the
reference's pure-PyTorch path:

* ``common/model.py``      RMSNorm, RoPE table and rotate-half, the layer, the head;
* ``solutions/packed.py``  the ragged packed forward (one rule for every token: a query
                           at position p of cache row r reads positions <= p of row r
                           after this call's K/V were written);
* ``common/engine.py`` / ``solutions/engine.py``  greedy AR and draft/verify drivers.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference and writes
``tests/golden/*.npz``); ``tests/test_oracle.py`` checks the pin.
"""
