"""CPU oracle for the DevProc compiled-pipeline path — TEST INFRASTRUCTURE.

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package; the product (``devproc_b200``) never
does.  It restates, on the CPU, what each IR op computes in the reference:

* ``interp.run_function`` — an IR interpreter, one torch-CPU function per IR
  op, each citing the reference call site that defines the op;
* ``preproc_np`` — a numpy restatement of the bilinear resize arithmetic of
  torch's CPU ``upsample_bilinear2d`` (the third-party function the
  reference's resize handler calls), used to pin the interpreter's resize;
* ``models`` — the seeded synthetic workloads of the benchmark configs.

Pinning: ``tests/golden/`` holds outputs of the reference's own Triton
templates, run on the CPU under ``TRITON_INTERPRET=1`` by
``tests/golden/make_golden.py``; ``tests/test_oracle.py`` checks this oracle
against them.
"""
