"""Stand-in for the ``visual_debug`` module that the reference's model glue
imports (manbo/gaussian_trace/model.py:10, render.py:15, legacy.py:5) but that
the reference repository does not contain.  Debug visualisation is off: the
hook records nothing and emit_visual_debug does nothing."""


class VisualDebugHook:
    def __init__(self, *args, **kwargs):
        self.enabled = False

    def __call__(self, *args, **kwargs):
        return None

    def __getattr__(self, name):
        return lambda *args, **kwargs: None


def emit_visual_debug(*args, **kwargs):
    return None


__all__ = ["VisualDebugHook", "emit_visual_debug"]
