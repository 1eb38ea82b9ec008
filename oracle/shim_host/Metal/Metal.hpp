// TEST INFRASTRUCTURE ONLY. A stand-in for the Metal part of Apple's metal-cpp
// (see Foundation/Foundation.hpp): buffers are zeroed host memory, pipelines
// and libraries are empty objects, and encoding or committing GPU work does
// nothing. Host code of the reference that only reads and writes buffer
// contents (its parameter init, act, actGreedy, setLogStd, lastStats, the
// slot accessors) therefore runs exactly as written; code that needs a GPU
// result gets none.
#pragma once

#include <cstdlib>
#include <cstring>

#include "../Foundation/Foundation.hpp"

namespace MTL {

using NS::UInteger;
enum ResourceOptions : UInteger { ResourceStorageModeShared = 0 };
enum CommandBufferStatus : UInteger { CommandBufferStatusCompleted = 4, CommandBufferStatusError = 5 };

struct Size {
    UInteger width, height, depth;
    Size(UInteger w, UInteger h, UInteger d) : width(w), height(h), depth(d) {}
};

class Buffer : public NS::Object {
   public:
    explicit Buffer(UInteger n) : bytes(n), data(std::calloc(n ? n : 1, 1)) {}
    ~Buffer() override { std::free(data); }
    void* contents() { return data; }
    UInteger length() const { return bytes; }
    UInteger bytes;
    void* data;
};

class Function : public NS::Object {};

class Library : public NS::Object {
   public:
    Function* newFunction(NS::String* name) {
        if (name) name->release();
        return new Function;
    }
};

class ComputePipelineState : public NS::Object {
   public:
    UInteger maxTotalThreadsPerThreadgroup() const { return 1024; }
};

class ComputeCommandEncoder : public NS::Object {
   public:
    void setComputePipelineState(ComputePipelineState*) {}
    void setBuffer(Buffer*, UInteger, UInteger) {}
    void setBytes(const void*, UInteger, UInteger) {}
    void dispatchThreads(Size, Size) {}
    void dispatchThreadgroups(Size, Size) {}
    void endEncoding() { delete this; }
};

class BlitCommandEncoder : public NS::Object {
   public:
    void fillBuffer(Buffer*, NS::Range, uint8_t) {}
    void copyFromBuffer(Buffer*, UInteger, Buffer*, UInteger, UInteger) {}
    void endEncoding() { delete this; }
};

class CommandBuffer : public NS::Object {
   public:
    ComputeCommandEncoder* computeCommandEncoder() { return new ComputeCommandEncoder; }
    BlitCommandEncoder* blitCommandEncoder() { return new BlitCommandEncoder; }
    void commit() {}
    void waitUntilCompleted() {}  // autoreleased in Metal: the caller never frees it (a few bytes leak here)
    CommandBufferStatus status() const { return CommandBufferStatusCompleted; }
    NS::Error* error() const { return nullptr; }
};

class CommandQueue : public NS::Object {
   public:
    CommandBuffer* commandBuffer() { return new CommandBuffer; }
};

class Device : public NS::Object {
   public:
    CommandQueue* newCommandQueue() { return new CommandQueue; }
    Library* newDefaultLibrary() { return new Library; }
    Buffer* newBuffer(UInteger bytes, ResourceOptions) { return new Buffer(bytes); }
    ComputePipelineState* newComputePipelineState(Function*, NS::Error**) { return new ComputePipelineState; }
};

inline Device* CreateSystemDefaultDevice() { return new Device; }

}  // namespace MTL
