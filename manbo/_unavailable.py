"""Placeholders for reference subsystems outside the B200 hot path."""


def unavailable(name: str, why: str = "outside the B200 render/optimise hot path"):
    def _fn(*args, **kwargs):
        raise NotImplementedError(f"{name} is not provided by the B200 build ({why})")
    _fn.__name__ = name
    _fn.__qualname__ = name
    return _fn


class UnavailableClass:
    _name = "object"

    def __init__(self, *args, **kwargs):
        raise NotImplementedError(
            f"{self._name} is not provided by the B200 build (outside the render/optimise hot path)")


def unavailable_class(name: str):
    return type(name, (UnavailableClass,), {"_name": name})
