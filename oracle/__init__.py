"""ORACLE — test infrastructure, not product.

CPU restatements of the reference's algorithms on the tensor-parallel forward path,
used only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` as the checker / the timed reference. Nothing in ``pyre_b200`` imports it.

* ``oracle.q80``      — Q8_0 quantize/dequantize (src/orchestrator/quantizer.py:11-40).
* ``oracle.kernels``  — pyre_kernels.mojo loops (rms_norm, softmax, apply_rope, silu_mul,
                        matmul_f32, q80_dequantize).
* ``oracle.ffn``      — FFN shard graph (src/ffn/builder.py:20-53) and the root/worker
                        decode FFN + partial sum (src/orchestrator/root_node.py:956-995,
                        src/orchestrator/worker_node.py:59-69, :319-329).
* ``oracle.partition``— solve_partitions (src/partitioner/solver.mojo:30-52),
                        AdaptivePartitioner / detect_drift (src/orchestrator/cluster.py:217-403).
* ``oracle/csrc``     — C restatement of the Mojo scalar loops and of the Q8_0 quantizer,
                        built into ``oracle/liboracle.so`` (CPU baseline and second checker).

Pinning: ``tests/golden/make_golden.py`` imports the reference's own ``quantizer.py`` and
runs its own ``ffn/builder.py`` (with a numpy stand-in for the absent MAX engine) to write
the fixtures in ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle
against them bit for bit (Q8_0) and to 1e-6 (FFN partials).
"""
