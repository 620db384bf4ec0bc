"""Evaluation harness: synthetic traces, an HTTP replay client that measures
TTFT / TBT per request, and a report over its results (and over a server's
telemetry directory). Reference roles: ``eval-tp/auto_benchmark_tp.py``
(timeline replay), ``eval-tp/compare_runs.py`` (A/B), ``scripts/timelines/``
(trace generators), ``scripts/metrics_report.py``."""
