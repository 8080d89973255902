"""CPU oracle for the quantized MoE expert hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (``tinyserve_b200``)
may import, call or link anything in this directory; only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` use it, and there only as the checker or as the timed
reference CPU path, never as the thing measured for the GPU arm.

Contents (each function cites the tinyserve file:line it restates):

- ``dequant``      numpy restatement of ``tinyserve/gguf_dequant_torch.py``
                   (``dequant_tensor``) and ``tinyserve/mxfp4.py``
                   (``dequant_mxfp4_no_transpose``), bit-exact.
- ``expert``       fp32 expert math (gate/up, SiLU or clamp-SwiGLU, down),
                   router (top-k then softmax) and weighted combine.
- ``cpu_expert_port``  the reference's CPU expert path
                   (``tinyserve/cpu_expert.py`` ``CPUExpertForward``) restated
                   with torch CPU ``F.linear``; timed as the CPU baseline.

Parity is pinned: ``tests/golden/`` holds vectors produced by importing the
reference's own decoders (``tests/golden/make_golden.py``), and
``tests/test_oracle.py`` checks this oracle against them and against the
reference tests' known-answer values.
"""
