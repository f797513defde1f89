import numpy as np


class DType:
    float32 = np.float32
    float16 = np.float16
    bfloat16 = "bfloat16"
    int32 = np.int32
    int64 = np.int64
