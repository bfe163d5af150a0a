"""Worker runtime (one process per GPU ring member): control-plane client, claim/execute/report
loop, heartbeats, supervisor; and the TCP tensor plane used by CPU ranks and cross-host paths."""
