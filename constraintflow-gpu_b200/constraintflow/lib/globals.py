"""Mode flags, device mode and JIT-capture store used by ConstraintFlow's generated code.

Same names as the reference's constraintflow/lib/globals.py (Flag :58-76, the mode flags
:83-92, DeviceMode :96-131, save_capture :35-55).  This runtime runs every tensor op on the
GPU, so the device mode is fixed to CUDA; the capture store is kept for programs compiled
in simulacrum mode.
"""
import json
import os

jit_root = "jit_captures"
_jit_store = {}


def set_jit_root(path):
    global jit_root
    jit_root = path


def jit_path(*parts):
    return os.path.join(jit_root, *parts)


def jit_store_clear():
    _jit_store.clear()


class Flag:
    def __init__(self):
        self.flag = False

    def set_flag(self):
        self.flag = True

    def reset_flag(self):
        self.flag = False

    def get_flag(self):
        return self.flag

    def __bool__(self):
        return self.flag

    def __str__(self):
        return f"flag: {self.flag}"


debug_flag = Flag()
dummy_mode = Flag()
reuse_mode = Flag()
dense_default_mode = Flag()
inductor_mode = Flag()
no_barriers = Flag()
in_memory_captures = Flag()


def save_capture(rel_path, obj):
    if in_memory_captures:
        _jit_store[rel_path] = json.dumps(obj)
        return
    path = jit_path(rel_path)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        json.dump(obj, f)


def load_capture(rel_path):
    if in_memory_captures:
        return json.loads(_jit_store[rel_path])
    with open(jit_path(rel_path)) as f:
        return json.load(f)


def capture_exists(rel_path):
    if in_memory_captures:
        return rel_path in _jit_store
    return os.path.exists(jit_path(rel_path))


class DeviceMode:
    """The reference switches between cpu / cuda / mps; here every op runs on CUDA."""

    _DEVICE_MAP = {"cpu": "cuda", "gpu": "cuda", "gpumac": "cuda"}

    def __init__(self):
        self._device = "cuda"

    def set_cpu(self):
        self._device = "cuda"

    def set_gpu(self):
        self._device = "cuda"

    def set_gpumac(self):
        self._device = "cuda"

    def set_mode(self, mode):
        if mode not in self._DEVICE_MAP:
            raise ValueError(f"Unknown device mode '{mode}'. Choose from: {list(self._DEVICE_MAP)}")
        self._device = self._DEVICE_MAP[mode]

    def get_device(self):
        return self._device

    def is_accelerated(self):
        return True

    def sync(self):
        import torch
        torch.cuda.synchronize()


device_mode = DeviceMode()


class Time:
    """Accumulating wall-clock timer (the reference keeps ~60 of these, globals.py:133-260)."""

    def __init__(self):
        self.total_time = 0.0
        self.num_used = 0

    def update_total_time(self, t):
        self.total_time += t
        self.num_used += 1

    def just_update_total_time(self, t):
        self.total_time += t

    def update_op_time(self, t):
        self.total_time += t

    def update_num_used(self):
        self.num_used += 1
