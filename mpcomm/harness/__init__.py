"""Command-line harness: a target server that publishes buffers and an
initiator that drives correctness/performance runs against targets.

    python -m mpcomm.harness.target    --host-id ... --tcp-port ... --buffer-size ...
    python -m mpcomm.harness.initiator --targets host_id:addr:port --mode all
"""
