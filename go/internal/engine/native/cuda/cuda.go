//go:build cuda && cgo

// Package cuda implements engine.Engine on the B200 decode engine
// (libb2decode.so, declared in include/b2decode.h) through cgo.
//
// It is the drop-in for the pure-Go transformer engine
// (internal/engine/native/transformer): the same Load / Unload / Predict /
// PredictStream / Embed / TokenCount / ModelInfo / IsLoaded behaviour
// (transformer.go:215-510), with the forward pass, the KV cache and the
// greedy loop on the GPU.  What stays in Go is what the reference already
// keeps outside its forward pass: the GGUF metadata parse for the tokenizer
// (gguf.Parse), BPE encode / decode (bpe.Tokenizer), and the text form of the
// stop words.  Token ids cross the ABI, never text.
//
// Build (Go toolchain with cgo, the library built by
// `make -C ai-agent-framework_b200`):
//
//	CGO_CFLAGS=-I<repo>/include CGO_LDFLAGS="-L<repo>/ai-agent-framework_b200 -lb2decode" \
//	    go build -tags cuda ./...
//
// and select it in cmd/server/main.go where transformer.New is called:
//
//	eng = cuda.New(logger)
package cuda

/*
#cgo LDFLAGS: -lb2decode
#include <stdlib.h>
#include "b2decode.h"
*/
import "C"

import (
	"context"
	"fmt"
	"os"
	"runtime"
	"strings"
	"sync"
	"time"
	"unsafe"

	"go.uber.org/zap"

	"github.com/your-org/local-llm/internal/domain"
	"github.com/your-org/local-llm/internal/engine"
	"github.com/your-org/local-llm/internal/engine/native/bpe"
	"github.com/your-org/local-llm/internal/engine/native/gguf"
)

// defaultMaxGen is the generation limit when num_predict <= 0
// (transformer.go:339-342).
const defaultMaxGen = 256

// streamBuffer is the channel capacity of PredictStream (transformer.go:394).
const streamBuffer = 32

// Engine is the GPU engine.  One mutex serialises every call, as the Go
// engine does (transformer.go:96); PredictStream holds it until its
// goroutine ends.
type Engine struct {
	mu     sync.Mutex
	logger *zap.Logger

	model  *C.b2_model
	cfg    C.b2_config
	tok    *bpe.Tokenizer
	meta   *engine.ModelMeta
	loaded bool

	// ids whose decoded text contains one of the stop words of the last
	// request (the token-id form of isStopToken, transformer.go:1430-1437)
	stopKey string
	stopIDs []int32
}

// New returns an engine with no model loaded.
func New(logger *zap.Logger) *Engine {
	if logger == nil {
		logger = zap.NewNop()
	}
	return &Engine{logger: logger}
}

// call runs one ABI call with the goroutine pinned to its OS thread, so that
// b2_last_error (thread-local) describes this call's failure.
func call(what string, f func() C.int) error {
	runtime.LockOSThread()
	defer runtime.UnlockOSThread()
	rc := f()
	if rc == C.B2_OK {
		return nil
	}
	return fmt.Errorf("%s: %s (b2decode error %d)", what, C.GoString(C.b2_last_error()), int(rc))
}

// Load parses the GGUF for the tokenizer and metadata and uploads the model
// to the GPU (transformer.go:215-310).
func (e *Engine) Load(_ context.Context, modelPath string, opts engine.LoadOptions) error {
	e.mu.Lock()
	defer e.mu.Unlock()
	start := time.Now()
	if e.loaded {
		e.unloadLocked()
	}
	gf, err := gguf.Parse(modelPath)
	if err != nil {
		return fmt.Errorf("parse gguf: %w", err)
	}
	tok, err := bpe.NewFromGGUF(gf)
	if err != nil {
		return fmt.Errorf("tokenizer: %w", err)
	}
	var lo C.b2_load_opts
	lo.num_ctx = C.int32_t(opts.NumCtx)
	cpath := C.CString(modelPath)
	defer C.free(unsafe.Pointer(cpath))
	var m *C.b2_model
	if err := call("load", func() C.int { return C.b2_load(cpath, &lo, &m) }); err != nil {
		return err
	}
	var cfg C.b2_config
	if err := call("config", func() C.int { return C.b2_get_config(m, &cfg) }); err != nil {
		C.b2_free(m)
		return err
	}
	var size int64
	if st, err := os.Stat(modelPath); err == nil {
		size = st.Size()
	}
	quant := "Q8_0"
	if cfg.weight_type == 2 {
		quant = "Q4_0"
	}
	e.model, e.cfg, e.tok = m, cfg, tok
	e.meta = &engine.ModelMeta{
		Name:          modelPath,
		Path:          modelPath,
		Family:        C.GoString(&cfg.arch[0]),
		ParameterSize: fmt.Sprintf("%dM", estimateParams(cfg)/1_000_000),
		QuantLevel:    quant,
		ContextLength: int(cfg.max_seq_len),
		EmbeddingSize: int(cfg.hidden_size),
		FileSizeBytes: size,
	}
	e.stopKey, e.stopIDs = "", nil
	e.loaded = true
	e.logger.Info("model loaded on the GPU",
		zap.Duration("elapsed", time.Since(start)),
		zap.Int64("weight_bytes", int64(cfg.weight_bytes)),
		zap.Int("max_seq_len", int(cfg.max_seq_len)))
	return nil
}

// estimateParams counts the weights as the Go engine does (transformer.go:512-517).
func estimateParams(cfg C.b2_config) int {
	h, ff, l, v := int(cfg.hidden_size), int(cfg.intermediate_size), int(cfg.num_layers), int(cfg.vocab_size)
	perLayer := 4*h*h + 3*h*ff + 2*h
	return v*h + l*perLayer + v*h
}

// Unload releases the model and its device memory (transformer.go:312-322).
func (e *Engine) Unload() error {
	e.mu.Lock()
	defer e.mu.Unlock()
	e.unloadLocked()
	return nil
}

func (e *Engine) unloadLocked() {
	if e.model != nil {
		C.b2_free(e.model)
	}
	e.model, e.tok, e.meta, e.loaded = nil, nil, nil, false
	e.stopKey, e.stopIDs = "", nil
}

// sampleOpts maps the request options (already merged with the server
// defaults by sampler.Merge in the handler) onto the ABI's.
func sampleOpts(o domain.Options) C.b2_sample_opts {
	var so C.b2_sample_opts
	so.temperature = C.double(o.Temperature)
	so.top_k = C.int32_t(o.TopK)
	so.top_p = C.double(o.TopP)
	so.repeat_penalty = C.double(o.RepeatPenalty)
	so.num_predict = C.int32_t(o.NumPredict)
	so.seed = C.uint64_t(o.Seed)
	return so
}

// stopIDsFor returns the ids whose decoded text contains a stop word: a
// sampled id is a stop exactly when isStopToken(DecodeToken(id), stop) is
// true (transformer.go:1430-1437), so checking ids on the GPU side is the
// same test.  Cached for the last stop list.
func (e *Engine) stopIDsFor(stop []string) []int32 {
	if len(stop) == 0 {
		return nil
	}
	key := strings.Join(stop, "\x00")
	if key == e.stopKey {
		return e.stopIDs
	}
	var ids []int32
	for id := 0; id < e.tok.VocabSize(); id++ {
		text := e.tok.DecodeToken(id)
		for _, sw := range stop {
			if strings.Contains(text, sw) {
				ids = append(ids, int32(id))
				break
			}
		}
	}
	e.stopKey, e.stopIDs = key, ids
	return ids
}

func int32s(ids []int) []int32 {
	out := make([]int32, len(ids))
	for i, v := range ids {
		out[i] = int32(v)
	}
	return out
}

func ints(ids []int32) []int {
	out := make([]int, len(ids))
	for i, v := range ids {
		out[i] = int(v)
	}
	return out
}

// ptr32 is the address of the first element, or nil for an empty slice.
func ptr32(s []int32) *C.int32_t {
	if len(s) == 0 {
		return nil
	}
	return (*C.int32_t)(unsafe.Pointer(&s[0]))
}

// Predict runs the whole generation (transformer.go:325-382): BOS + prompt
// ids, prefill, then up to num_predict tokens, stopping at EOS or a stop word.
func (e *Engine) Predict(ctx context.Context, req domain.InferenceRequest) (engine.PredictResult, error) {
	e.mu.Lock()
	defer e.mu.Unlock()
	if !e.loaded {
		return engine.PredictResult{}, fmt.Errorf("no model loaded")
	}
	if err := ctx.Err(); err != nil {
		return engine.PredictResult{}, err
	}
	start := time.Now()
	prompt := int32s(e.tok.Encode(req.Prompt))
	stop := e.stopIDsFor(req.Options.Stop)
	maxOut := req.Options.NumPredict
	if maxOut <= 0 {
		maxOut = defaultMaxGen
	}
	out := make([]int32, maxOut)
	so := sampleOpts(req.Options)
	var n C.int32_t
	var tm C.b2_timings
	err := call("predict", func() C.int {
		return C.b2_predict(e.model, ptr32(prompt), C.int32_t(len(prompt)), &so, ptr32(stop), C.int32_t(len(stop)),
			ptr32(out), C.int32_t(maxOut), &n, &tm)
	})
	if err != nil {
		return engine.PredictResult{}, err
	}
	gen := ints(out[:int(n)])
	return engine.PredictResult{
		Text:             e.tok.Decode(gen),
		PromptTokens:     int(tm.prompt_tokens),
		CompletionTokens: len(gen),
		TotalDuration:    time.Since(start).Nanoseconds(),
		PromptDuration:   int64(tm.prompt_ns),
		EvalDuration:     int64(tm.eval_ns),
	}, nil
}

// PredictStream streams one token at a time (transformer.go:385-442): the
// channel (buffer 32) is closed by the engine, its last item has Done set,
// and an error arrives as StreamToken{Err, Done: true}.  The engine stays
// locked until the goroutine ends.
func (e *Engine) PredictStream(ctx context.Context, req domain.InferenceRequest) (<-chan engine.StreamToken, error) {
	e.mu.Lock()
	if !e.loaded {
		e.mu.Unlock()
		return nil, fmt.Errorf("no model loaded")
	}
	prompt := int32s(e.tok.Encode(req.Prompt))
	stop := e.stopIDsFor(req.Options.Stop)
	so := sampleOpts(req.Options)
	if err := call("stream begin", func() C.int {
		return C.b2_stream_begin(e.model, ptr32(prompt), C.int32_t(len(prompt)), &so, ptr32(stop), C.int32_t(len(stop)))
	}); err != nil {
		e.mu.Unlock()
		return nil, err
	}
	ch := make(chan engine.StreamToken, streamBuffer)
	go func() {
		defer close(ch)
		defer e.mu.Unlock()
		for {
			if err := ctx.Err(); err != nil {
				ch <- engine.StreamToken{Err: err, Done: true}
				return
			}
			var id, done C.int32_t
			if err := call("stream next", func() C.int { return C.b2_stream_next(e.model, &id, &done) }); err != nil {
				ch <- engine.StreamToken{Err: err, Done: true}
				return
			}
			if done != 0 {
				ch <- engine.StreamToken{Done: true}
				return
			}
			ch <- engine.StreamToken{Text: e.tok.DecodeToken(int(id))}
		}
	}()
	return ch, nil
}

// Embed returns the mean of each text's token embeddings, L2-normalised
// (transformer.go:445-490); an empty text embeds to zeros.
func (e *Engine) Embed(_ context.Context, texts []string) ([][]float32, error) {
	e.mu.Lock()
	defer e.mu.Unlock()
	if !e.loaded {
		return nil, fmt.Errorf("no model loaded")
	}
	h := int(e.cfg.hidden_size)
	results := make([][]float32, len(texts))
	for i, text := range texts {
		ids := int32s(e.tok.Encode(text))
		vec := make([]float32, h)
		if len(ids) > 0 {
			err := call("embed", func() C.int {
				return C.b2_embed(e.model, ptr32(ids), C.int32_t(len(ids)), (*C.float)(unsafe.Pointer(&vec[0])))
			})
			if err != nil {
				return nil, err
			}
		}
		results[i] = vec
	}
	return results, nil
}

// TokenCount is the number of prompt ids of the text (no BOS), as the Go
// engine counts them (transformer.go:492-499).
func (e *Engine) TokenCount(_ context.Context, text string) (int, error) {
	e.mu.Lock()
	defer e.mu.Unlock()
	if !e.loaded {
		return 0, fmt.Errorf("no model loaded")
	}
	return len(e.tok.Encode(text)), nil
}

// ModelInfo returns the loaded model's metadata, nil when none is loaded.
func (e *Engine) ModelInfo() *engine.ModelMeta {
	e.mu.Lock()
	defer e.mu.Unlock()
	return e.meta
}

// IsLoaded reports whether a model is loaded.
func (e *Engine) IsLoaded() bool {
	e.mu.Lock()
	defer e.mu.Unlock()
	return e.loaded
}

var _ engine.Engine = (*Engine)(nil)
