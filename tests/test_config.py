

def test_log_level_switch(monkeypatch):
    import logging

    from gollek_b200.utils.log import configure_logging
    monkeypatch.setenv("GOLLEK_LOG_LEVEL", "off")
    log = configure_logging()
    assert not log.isEnabledFor(logging.CRITICAL)
    assert configure_logging("debug").isEnabledFor(logging.DEBUG)
    assert sum(getattr(h, "_gollek", False) for h in log.handlers) == 1
    import pytest
    with pytest.raises(ValueError):
        configure_logging("loud")
