"""Timers, seeding and device-side phase timing."""

from .timers import DeviceTimers, Timer, Timers, set_seed

__all__ = ["Timer", "Timers", "DeviceTimers", "set_seed"]
