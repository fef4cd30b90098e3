"""CPU oracle of the testt_b200 hot path. TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference (SalReII/testt, `solution/`)
for every op of the path; each function cites the reference file:line it follows. It is the
checker: only `tests/`, `__graft_entry__.smoke()` and `bench.py` (its `cpu_baseline` leg and its
`--impl reference` arm) may import it. The product (`testt_b200/`) never imports, links or runs
anything from here.

Pinning: `tests/golden/*.npz` hold inputs and outputs of the reference's own Triton kernels, run
on the CPU through Triton's interpreter (`tests/golden/make_golden.py`); `tests/test_oracle.py`
checks this oracle against them (bit-exact for NF4, within the kernels' tolerances otherwise).

- `nf4`     NF4 code table (QLoRA construction), quantiser (plain and nested absmax), dequantiser
- `ops`     fp32/fp64 torch restatements of add+RMSNorm, RoPE pack, gated SiLU and the head
- `synth`   seeded synthetic inputs of the benchmark configurations
- `nf4_ref.c` the NF4 dequantiser in C (OpenMP), used as the timed CPU baseline
"""
