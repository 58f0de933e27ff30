"""L8 fault injection: in-worker hook-point injector and host-level external injector."""
