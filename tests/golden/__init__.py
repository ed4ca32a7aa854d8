"""Golden vectors for the attention path: seeded cases (cases.py), their
outputs from the reference's own compiled kernels (golden.npz), and the
script that made them (make_golden.py)."""
