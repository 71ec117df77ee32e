"""Command-line entry points: training and generation runtimes, launch planning."""
