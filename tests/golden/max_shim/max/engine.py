import numpy as np

from .driver import Tensor

# The reference compiles its root FFN graph for a fixed 64-token prefill (root_node.py:143-151)
# and pads every prompt to that length. Fixture scripts that drive longer prompts set this to
# True: inputs may then differ from the declared type in the sequence dim (axis 1) only. The
# graph's ops (matmul, silu, mul) act on each token row independently, so a row's result does
# not depend on the sequence length.
ANY_SEQ_LEN = False


class _Model:
    def __init__(self, graph):
        self.graph = graph

    def execute(self, *arrays):
        env = {"inputs": [np.asarray(a) for a in arrays]}
        for a, t in zip(env["inputs"], self.graph.input_types):
            want = list(t.shape)
            got = list(a.shape)
            if ANY_SEQ_LEN and len(got) == 3 and len(want) == 3:
                got[1] = want[1]
            if got != want:
                raise ValueError(f"input shape {a.shape} != graph type {t.shape}")
        return tuple(Tensor(o.eval(env)) for o in self.graph.outputs)


class InferenceSession:
    def __init__(self, devices=None):
        self.devices = devices

    def load(self, graph):
        return _Model(graph)
