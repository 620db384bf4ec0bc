"""Adapter management: PEFT checkpoint I/O and adapter routing."""
