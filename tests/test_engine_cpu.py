"""Host-side logic of the engine that needs no GPU: every method that
launches kernels runs with the engine's own device current."""

import contextlib
import types

from diffusionhard_b200 import engine as engine_mod

LAUNCHING = ("forward", "final_hidden_q", "logits", "selected_logits", "head_argmax", "enqueue_transition",
             "init_loop", "generate", "generate_event_driven", "_load_schedule")


def test_launching_methods_are_pinned_to_the_engine_device():
    for name in LAUNCHING:
        assert hasattr(getattr(engine_mod.MDLMEngine, name), "__wrapped__"), name


def test_pinned_method_enters_the_engine_device():
    seen = []

    @contextlib.contextmanager
    def device(d):
        seen.append(("enter", d))
        yield
        seen.append(("exit", d))

    fake = types.SimpleNamespace(torch=types.SimpleNamespace(cuda=types.SimpleNamespace(device=device)),
                                 device="cuda:1")

    @engine_mod._on_device
    def launch(self, value):
        seen.append(("body", value))
        return value + 1

    assert launch(fake, 41) == 42
    assert seen == [("enter", "cuda:1"), ("body", 41), ("exit", "cuda:1")]

