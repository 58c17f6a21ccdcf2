"""Run by tests/test_reference_suite.py in a pytest child with `-p refshim` and KUSHKASH_PAGE=16 (not collected on its
own): the unmodified kushkash SGLang plugin declares and sizes 16-token pages once the drop-in is installed at page
16.  The SGLang classes the plugin subclasses are the reference test file's own stand-ins (kushkash's
tests/test_sglang_backend_cpu.py, `_stub_modules`); SGLang itself is not installed here."""
import sys
import types

import pytest
import torch

pytestmark = pytest.mark.skipif(__import__("os").environ.get("KUSHKASH_PAGE") != "16", reason="page-16 run only")


def test_page_constants():
    import kushkash
    import kushkash._ops as ops
    import kushkash.cache as cache
    import kushkash.sglang as ks
    import kushkash_b200.dropin as dropin
    assert dropin.page() == 16 and ops.PAGE == cache.PAGE == ks.PAGE == kushkash.PAGE == 16
    assert ops.record_bytes(128, 4) == 2624 and ops.record_bytes(128, 8) == 4672
    cfg = kushkash._build.GpuConfig(128, 4, 4, "bfloat16", "sm_100")
    assert cfg.page == 16


def test_sglang_declares_page_16():
    import enum
    import kushkash.sglang as ks

    class Backend(enum.Enum):
        DISABLED = "disabled"
        FULL = "full"

    class Phase(enum.Enum):
        PREFILL = "prefill"

    def with_phase(cfg, phase, backend):
        return (phase, backend)

    def cfg(**kw):
        base = dict(attention_backend="kushkash", prefill_attention_backend=None, decode_attention_backend=None,
                    kv_cache_dtype="auto", speculative_algorithm=None, page_size=None, max_running_requests=None,
                    cuda_graph_config=types.SimpleNamespace(prefill=types.SimpleNamespace(backend=Backend.DISABLED)))
        base.update(kw)
        return types.SimpleNamespace(**base)

    assert ks.server_args_decisions(cfg(), (), Backend, Phase, with_phase)["page_size"] == 16
    assert ks.server_args_decisions(cfg(page_size=32), (), Backend, Phase, with_phase)["page_size"] == 16
    assert ks.server_args_decisions(cfg(page_size=16, max_running_requests=64), (), Backend, Phase, with_phase) == {}
    # the exact-K tail the budget hook reserves: one 16-token page per request slot, kv head and layer
    assert ks.tail_bytes(257, 32, 8, 128, 2) == 257 * 32 * 8 * 16 * 128 * 2


def test_sglang_pool_holds_16_token_records(monkeypatch):
    import test_sglang_backend_cpu as ref                  # the reference's stand-ins for the SGLang base classes
    with pytest.MonkeyPatch.context() as mp:
        for name, mod in ref._stub_modules().items():
            mp.setitem(sys.modules, name, mod)
        ref._drop_backend_modules()
        from kushkash.sglang import pool
        monkeypatch.setenv("KUSHKASH_BITS", "4")
        p = pool.KushPool(size=100 * 16, page_size=16, head_num=2, head_dim=128, layer_num=3,
                          device=torch.device("cpu"))
        assert p.k_buffer[0].shape == (101, 2, 2624) and len(p.k_buffer) == 3
        with pytest.raises(ValueError, match="page_size 16"):
            pool.KushPool(size=100 * 32, page_size=32, head_num=2, head_dim=128, layer_num=1,
                          device=torch.device("cpu"))
        ref._drop_backend_modules()
