"""CPU oracle for noise_b200 — TEST INFRASTRUCTURE ONLY.

A plain restatement, in numpy and CPU torch, of the reference's forward-only ES step (Noise,
`train/val/eggroll.py`, `train/val/run.py`, `utils/model.py`), used to check the CUDA path.
Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU baseline arm may import it, and only
as the checker or the timed CPU baseline; the product path (`noise_b200`) never calls into it.

Parity pin: the restatement is checked against golden vectors produced by running the reference's
own functions on CPU in the build container (`tests/golden/make_golden.py`, fixtures committed in
`tests/golden/`).
"""
