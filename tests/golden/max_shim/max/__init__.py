"""Numpy stand-in for the Modular MAX packages the reference imports (max.graph,
max.engine, max.driver, max.dtype). Fixture generation only: it lets
tests/golden/make_golden.py run the reference's own Python (src/ffn/builder.py,
src/attention/builder.py, src/orchestrator/cluster.py) in this container, where MAX is not
installed. Graph ops evaluate in float32 numpy."""
