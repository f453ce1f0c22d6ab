"""CPU oracle for the integer-only SmolLM2-135M forward pass.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped engine imports, links or runs
anything under this directory; only tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py use it, and only as the checker.

Contents
  formats.json    per-layer (bits, f) activation formats, derived from the
                  reference's results/scaling_proposal.json by make_formats.py
  tables.py       exact mpmath tables (exp, SiLU, RoPE)
  synth.py        seeded synthetic float model -> quantised model.bin
  modelbin.py     model.bin reader/writer (c/intref.c:8-13 layout)
  forward.py      numpy restatement of python/intref.py (the definition)
  build_ref.sh    compiles the reference's own c/intref.c into oracle/_ref/

Parity pin: tests/golden/ holds sha256 digests of model.bin and of every
exported state produced by the reference's OWN python/intref.py +
python/export_vectors.py on the same seeded synthetic weights
(tests/golden/make_golden.py), and tests/test_oracle_golden.py checks this
restatement against them.
"""
