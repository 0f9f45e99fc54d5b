"""CPU oracle for the Atlas-RNN memory-update hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this folder.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg may import it, and only as the checker (or as the
timed CPU restatement of the reference), never as the product path.

Contents
--------
* ``assoc_scan_standin`` -- stand-in for the third-party ``assoc_scan`` package
  (PyPI "assoc-scan", unpinned in the reference's pyproject.toml:28 and absent
  from this image). Scalar-gate specialisation of the odd/even recursive scan of
  ``atlas_pytorch/affine_scan.py:102-137``.
* ``memory_ref`` -- restatement of the reference recurrence core
  (``atlas_pytorch/rnn_memory.py:345-393`` Titans, ``:655-717`` Omega) at the
  q/k/v/gates boundary, in torch CPU ops (float64 by default) so autograd gives
  every input gradient exactly as the reference's own autograd does; plus a
  sequential float64 numpy restatement used to cross-check it.
* ``harness`` -- module-substitution harness that drives the reference's own
  ``_forward_impl`` (only usable where the reference sources exist; used by
  ``tests/golden/make_golden.py`` to pin this oracle).

Parity pinning: the oracle is checked against golden vectors produced by the
reference module itself (``tests/golden/*.npz``) and against the reference
tests' known-answer cases (scan / window KATs, split-scan identity).
"""
