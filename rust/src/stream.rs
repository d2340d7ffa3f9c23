//! Incremental UTF-8 output of sampled tokens, one buffer per row of a batch (host side).
//!
//! rust-llama's `ByteStream` (src/main.rs:829-867) and its server's generation core
//! (src/server.rs:186-215) append each token's bytes to a pending buffer, emit the longest valid
//! UTF-8 prefix and keep the rest; the remainder is emitted lossily at the end.  `ByteStreams`
//! keeps one such buffer per row of a batched generation loop; the token -> bytes mapping is the
//! caller's tokenizer.

/// One sequence's pending bytes.
#[derive(Default, Debug, Clone)]
pub struct ByteStream {
    pending: Vec<u8>,
}

impl ByteStream {
    /// Appends a token's bytes and returns the text that became complete.
    pub fn push(&mut self, token_bytes: &[u8]) -> String {
        self.pending.extend_from_slice(token_bytes);
        let valid = match std::str::from_utf8(&self.pending) {
            Ok(s) => s.len(),
            Err(e) => e.valid_up_to(),
        };
        let out = String::from_utf8(self.pending[..valid].to_vec()).unwrap_or_default();
        self.pending.drain(..valid);
        out
    }

    /// The remaining bytes, lossily.
    pub fn flush(&mut self) -> String {
        let out = String::from_utf8_lossy(&self.pending).into_owned();
        self.pending.clear();
        out
    }
}

/// One `ByteStream` per row.
#[derive(Default, Debug, Clone)]
pub struct ByteStreams {
    streams: Vec<ByteStream>,
}

impl ByteStreams {
    pub fn new(rows: usize) -> Self {
        ByteStreams { streams: vec![ByteStream::default(); rows] }
    }

    /// The text each row's new token completes (rows whose `active` entry is false: empty).
    pub fn push<F: Fn(u32) -> Vec<u8>>(&mut self, tokens: &[u32], active: &[bool], token_bytes: F) -> Vec<String> {
        self.streams
            .iter_mut()
            .zip(tokens.iter().zip(active.iter()))
            .map(|(s, (&t, &a))| if a { s.push(&token_bytes(t)) } else { String::new() })
            .collect()
    }

    pub fn flush(&mut self) -> Vec<String> {
        self.streams.iter_mut().map(|s| s.flush()).collect()
    }
}
