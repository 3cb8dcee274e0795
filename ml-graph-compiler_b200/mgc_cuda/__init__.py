"""B200 (sm_100a) `cuda` target for ml-graph-compiler."""
