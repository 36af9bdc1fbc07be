"""Handle release order of the Python binding (no GPU: a fake library
records the C calls). A context releases the sessions, models and weights
that live in it before it is destroyed, a model its sessions before itself,
and a handle whose context is already gone is dropped without a C call (the
C side would otherwise touch freed memory)."""
import unltd_gpu as ug


class _FakeLib:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def f(*a):
            self.calls.append((name, a[0] if a else None))
            return 0
        return f


def _objects():
    c = object.__new__(ug.Context)
    c.h = "C"
    w = ug.Weight(c, "W", ug.Q4K, 256, 1)
    m = object.__new__(ug.Qwen35Model)
    m.ctx, m.h = c, "M"
    ug._track(m, 1)
    s = ug.Qwen35Session(m, "S", 16)
    return c, w, m, s


def test_context_close_releases_its_handles_first(monkeypatch):
    fake = _FakeLib()
    monkeypatch.setattr(ug, "_lib", fake)
    c, w, m, s = _objects()
    c.close()
    assert fake.calls == [("unltd_qwen35_session_destroy", "S"), ("unltd_qwen35_destroy", "M"),
                          ("unltd_weight_free", "W"), ("unltd_ctx_destroy", "C")]
    # closing again (e.g. at interpreter exit) makes no further C calls
    w.free(), s.close(), m.close(), c.close()
    assert len(fake.calls) == 4


def test_model_close_releases_its_sessions_first(monkeypatch):
    fake = _FakeLib()
    monkeypatch.setattr(ug, "_lib", fake)
    c, w, m, s = _objects()
    m.close()
    assert fake.calls == [("unltd_qwen35_session_destroy", "S"), ("unltd_qwen35_destroy", "M")]
    s.close()
    assert len(fake.calls) == 2
    c.close()
    assert fake.calls[2:] == [("unltd_weight_free", "W"), ("unltd_ctx_destroy", "C")]


def test_handle_of_a_destroyed_context_is_dropped(monkeypatch):
    fake = _FakeLib()
    monkeypatch.setattr(ug, "_lib", fake)
    c, w, m, s = _objects()
    c.h = None  # context destroyed behind the handles' backs
    w.free(), s.close(), m.close()
    assert fake.calls == [] and w.h is None and s.h is None and m.h is None
