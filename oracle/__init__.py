"""TEST INFRASTRUCTURE ONLY — the parity oracle of the attention hot path.

`oracle.cpu` is the fp32 C restatement of the reference kernels (attn_ref.c -> liboracle.so, numpy in/out).
`oracle.refkern` launches the reference's own kernels (kernels/voxcpm.cu built to oracle/_ref/voxcpm_ref.fatbin as
compute_80 PTX, JIT-compiled by the driver) with the reference's launch shapes.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use this package.
"""
