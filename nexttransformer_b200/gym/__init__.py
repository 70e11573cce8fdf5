"""Research gym: an HTTP / MCP service for agent-driven architecture research on this framework.

Candidates are source-only method plugins; their cost is the audited FLOP ledger's; experiments
run in isolated worker processes on leased GPUs under a FLOP budget (``contract``, ``package``,
``store``, ``resources``, ``research``, ``worker``, ``service``, ``client``, ``mcp``).
"""
