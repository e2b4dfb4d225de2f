"""Oracle: CPU restatement of torch-sla's iterative-solve hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (torch_sla_b200/) imports
this package; only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs use it, and only as the checker / the timed CPU reference.

* krylov.py    -- PCG, PBiCGStab, batched same-pattern CG, the adjoint
                  gradients and the Shard(0) CG/BiCGStab control flow, written
                  on the same PyTorch CPU ops (ATen: sparse CSR torch.mv,
                  torch.vdot, addcmul) that torch-sla's `pytorch` backend
                  calls, so its arithmetic is the reference's arithmetic.
                  ATen is a third-party dependency of torch-sla (pinned only
                  as torch>=1.10.0 in its pyproject.toml; torch 2.11.0 here).
* partition.py -- numpy restatement of partition_simple / find_halo_nodes /
                  build_partition / extract_partition (integer maps,
                  compared bit-exactly).

Pinning: tests/golden/make_golden.py runs the reference itself (imported from
its source tree in the build container) on seeded inputs and stores the
outputs under tests/golden/; tests/test_oracle_golden.py checks this oracle
against those fixtures.
"""
