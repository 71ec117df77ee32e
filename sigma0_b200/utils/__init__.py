"""Utilities: config reader, timers, watchdog, FLOP counting."""
