import numpy as np


class DeviceRef:
    def __init__(self, kind="cpu", id=0):
        self.kind, self.id = kind, id

    @staticmethod
    def CPU(id=0):
        return DeviceRef("cpu", id)

    @staticmethod
    def GPU(id=0):
        return DeviceRef("gpu", id)


class TensorType:
    def __init__(self, dtype, shape, device=None):
        self.dtype, self.shape, self.device = dtype, list(shape), device


class _Node:
    def __init__(self, fn, args):
        self.fn, self.args = fn, args

    def eval(self, env):
        if id(self) in env:
            return env[id(self)]
        v = self.fn(*[a.eval(env) if isinstance(a, _Node) else a for a in self.args])
        env[id(self)] = v
        return v

    def __mul__(self, other):
        return _Node(lambda a, b: (a * b).astype(np.float32), [self, other])

    def __add__(self, other):
        return _Node(lambda a, b: (a + b).astype(np.float32), [self, other])


class _Input(_Node):
    def __init__(self, idx):
        super().__init__(None, [])
        self.idx = idx

    def eval(self, env):
        return env["inputs"][self.idx]


class Graph:
    def __init__(self, name, input_types=()):
        self.name = name
        self.input_types = list(input_types)
        self.inputs = [_Input(i) for i in range(len(self.input_types))]
        self.outputs = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def output(self, *nodes):
        self.outputs = list(nodes)


class ops:
    @staticmethod
    def matmul(a, b):
        return _Node(lambda x, y: np.matmul(x.astype(np.float32), y.astype(np.float32)).astype(np.float32), [a, b])

    @staticmethod
    def silu(a):
        def f(x):
            x = x.astype(np.float32)
            with np.errstate(over="ignore"):
                return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)
        return _Node(f, [a])

    @staticmethod
    def reshape(a, shape):
        return _Node(lambda x: x.reshape(shape), [a])
