def cast_to(weight, dtype=None, device=None, non_blocking=False, copy=False, stream=None):
    return weight.to(device=device, dtype=dtype if dtype is not None else weight.dtype)
