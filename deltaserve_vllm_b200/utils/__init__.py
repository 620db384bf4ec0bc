"""Run telemetry (metrics recorder, step trace) and the offline tokenizer."""
