"""CPU oracle for the tidegs_b200 hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference (TideGS) algorithms that
libtidegs_b200.so implements on the GPU. It exists to check the product,
never to be the product: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg / reference arm may import it. Nothing in tidegs_b200/
imports it.

Pinning: each module states how it is pinned. The resident-Adam, block
materialization, write-back pack, bounds and dirty-bitmap restatements are
checked against golden vectors produced by running the reference's own CPU
code paths (tests/golden/make_golden.py). The SelectiveAdam restatement
follows submodules/clm_kernels/adam.cu and is checked against that kernel
compiled from the reference sources (oracle/build_ref.py) where a GPU is
available. The touched-only gradient accumulation (sparse_grad.py) is
checked against the reference's own torch operations run on the CPU. The
Sophia restatement has no reference implementation in TideGS: parity
unpinned.
"""
